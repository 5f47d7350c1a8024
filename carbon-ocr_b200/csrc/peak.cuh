// The tensor cores' dense rate on this GPU, measured: one CTA a SM, one thread issuing
// back-to-back tcgen05.mma (M = 128, K = 32 bytes, N given) from a shared-memory tile into one
// TMEM accumulator, nothing else.  The roofline's denominator for the INT8 and FP16 kernels
// (the driver measures only BF16 through cuBLAS), and the per-instruction cost at each N.
#pragma once

#include <cstdint>

#include "sm100.cuh"

namespace crec {

constexpr int kPeakSmem = 160 << 10;  // more than half an SM's shared memory: one CTA a SM

template <bool kInt8>
__global__ void __launch_bounds__(128, 1) mma_peak_kernel(int n, int iters, int* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a = smem;            // [128][128] bytes
  uint8_t* b = smem + 16384;    // [n][128] bytes
  uint64_t* done = reinterpret_cast<uint64_t*>(b + 256 * 128);
  uint32_t* slot = reinterpret_cast<uint32_t*>(done + 1);
  for (int i = threadIdx.x; i < (16384 + n * 128) / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
  fence_proxy_async_smem();  // the zeros, written by threads, before the tensor core reads them
  if (threadIdx.x == 0) {
    mbar_init(done, 1);
    fence_mbar_init();
  }
  if (threadIdx.x < 32) tmem_alloc(slot, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *slot;
  if (threadIdx.x == 0) {
    const uint32_t idesc = kInt8 ? idesc_i8(n) : idesc_f16(n);
    const uint64_t ad = umma_desc_sw128(smem_u32(a)), bd = umma_desc_sw128(smem_u32(b));
    for (int i = 0; i < iters; ++i) {
#pragma unroll
      for (int s = 0; s < 4; ++s) umma<kInt8>(tmem, ad + 2 * s, bd + 2 * s, idesc, (i | s) ? 1u : 0u);
    }
    umma_commit(done);
    mbar_wait(done, 0, err, kErrTimeoutFull);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x < 32) tmem_dealloc(tmem, 256);
}

}  // namespace crec
