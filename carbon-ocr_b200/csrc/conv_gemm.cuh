// Dense convolutions (3x3, 2x3, 1x1, any stride) as implicit GEMMs on the fifth-generation
// tensor cores: tcgen05.mma with the accumulators in TMEM, operands staged in shared memory by
// TMA, one persistent CTA per SM.
//
// The GEMM: rows are output pixels, 128 consecutive columns of one output row a tile; columns
// are output channels (a tile of at most 256); K is (kernel row, kernel column, input channel).
// A tensor is NHWC with its channels padded to a multiple of 16 bytes, and a whole group of
// lines lies end to end along its width, each line's columns separated by gap columns that
// hold the zero point (the borders the reference keeps around every tensor,
// carbon/src/net/net.cpp:100-160).  For kernel row ky, the kw * C bytes a pixel's taps read in
// that row are contiguous, and successive output columns' windows start sw * C bytes apart:
// a 3-d tensor map over (window byte, output column, output row) with those strides is the
// im2col of the layer, so each stage is one TMA box of 128 window bytes x 128 pixels into
// the 128-byte swizzle that the MMA reads.  Weights are pre-arranged on the host in the same
// swizzled image and arrive by one bulk copy a stage.
//
// INT8: A is uint8 (the activation), B int8 (the weights); the MMA's sum of a * w minus
// zero * sum(w) is the reference's sum of (a - zero) * w (carbon/src/cpu/kernels.cpp:140-154),
// exact in int32.  The epilogue is the reference's output stage (carbon/src/cpu/kernels.h:354-380)
// operation by operation, each rounded on its own: sum * scale, + bias, + (residual - rz) * rs,
// ReLU, * inv_scale, clamped to [-zero, 255 - zero], rounded half to even, + zero.
// FP16: A and B float16, FP32 sums; bias, residual and ReLU in FP32, stored as float16.
//
// Warp roles (10 warps): 0 TMA producer, 1 MMA issuer (and TMEM owner), 2-9 epilogue: two warps
// for each TMEM lane quarter (the quarter of its warp index mod 4), each taking half of a tile's
// channel groups.  The epilogue is where an INT8 layer's time goes (requantizing 128 x N outputs
// costs more CUDA-core cycles than the tensor cores' MMAs for K below ~700), hence 8 warps, the
// per-channel constants in shared memory, and for layers with both zero points 0 and a ReLU
// (most of the backbone) one saturating convert: cvt.rni.sat.u8 rounds half to even and clamps
// to [0, 255], which is the reference's ReLU, clamp and round for a zero point of 0.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "crop_stem.cuh"  // cvt_rni_sat_u8
#include "sm100.cuh"

namespace crec {

struct ConvParams {
  CUtensorMap tmap[3];  // one per kernel row (kh <= 3)
  const uint8_t* wimg;  // [n tile][ky][kb][nt rows][128 bytes], each block in the 128-byte swizzle
  int kh, nkb, last_steps;  // K blocks of 128 bytes per kernel row; 32-byte K steps in each row's last block
  int nt, n_tiles;          // output channels a tile (multiple of 16, <= 256), tiles across the channels
  int oh, ow, m_per_row, num_tiles;
  int stages;
  uint32_t stage_bytes, a_bytes, b_bytes;
  // epilogue
  uint8_t* out;  // the output tensor's first row (its top border row)
  int out_ph;
  long long out_pitch;  // bytes per output row
  int cp_out, c_out, ebytes;
  const int32_t* colsum;  // [cp_out] sum of each output channel's int8 weights
  const float* scale;     // [cp_out] input scale * weight scale (int8)
  const float* bias;      // [cp_out]
  int in_zero, out_zero, relu;
  float out_inv_scale;
  const uint8_t* res;  // residual tensor's first row, or null
  int res_ph, res_cp, res_shift, res_zero;
  long long res_pitch;
  float res_scale;
  const uint8_t* mask8;  // one byte per 8 input columns: 1 where a line is
  int out_shift;         // log2 of input columns per output column
  int* err;
};

constexpr int kConvThreads = 320;
constexpr int kConvEpiWarps = 8;
constexpr uint32_t kTmemCols = 512;

template <bool kInt8>
__global__ void __launch_bounds__(kConvThreads, 1) conv_gemm_kernel(const __grid_constant__ ConvParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-aligned base for the swizzled stages
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.stages * p.stage_bytes);
  uint64_t* empty = full + p.stages;
  uint64_t* tmem_full = empty + p.stages;
  uint64_t* tmem_empty = tmem_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_empty + 2);
  int32_t* s_colsum = reinterpret_cast<int32_t*>(tmem_slot + 4);  // [cp_out] per-channel constants
  float* s_scale = reinterpret_cast<float*>(s_colsum + p.cp_out);
  float* s_bias = s_scale + p.cp_out;
  for (int j = threadIdx.x; j < p.cp_out; j += blockDim.x) {
    s_colsum[j] = p.colsum[j];
    s_scale[j] = p.scale[j];
    s_bias[j] = p.bias[j];
  }

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], kConvEpiWarps);
    }
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  if (warp == 0 && lane == 0) {
    for (int k = 0; k < p.kh; ++k) prefetch_tmap(&p.tmap[k]);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int ksteps_per_tile = p.kh * p.nkb;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
        const int n = t % p.n_tiles, m = t / p.n_tiles;
        const int oy = m / p.m_per_row, ox0 = (m % p.m_per_row) * 128;
        for (int ky = 0; ky < p.kh && ok; ++ky) {
          for (int kb = 0; kb < p.nkb; ++kb) {
            if (!mbar_wait(&empty[stage], phase ^ 1, p.err, kErrTimeoutEmpty)) {
              ok = false;
              break;
            }
            uint8_t* a = smem + stage * p.stage_bytes;
            uint8_t* b = a + p.a_bytes;
            mbar_expect_tx(&full[stage], p.a_bytes + p.b_bytes);
            tma_load_3d(a, &p.tmap[ky], kb * 128, ox0, oy, &full[stage]);
            const uint8_t* w = p.wimg + (static_cast<size_t>((n * p.kh + ky) * p.nkb + kb)) * p.b_bytes;
            bulk_load(b, w, p.b_bytes, &full[stage]);
            if (++stage == p.stages) {
              stage = 0;
              phase ^= 1;
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = kInt8 ? idesc_i8(p.nt) : idesc_f16(p.nt);
      int stage = 0;
      uint32_t phase = 0;
      int iter = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x, ++iter) {
        const int acc = iter & 1;
        const uint32_t acc_phase = (iter >> 1) & 1;
        if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1, p.err, kErrTimeoutTmemEmpty)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * 256);
        uint32_t accumulate = 0;
        for (int ks = 0; ks < ksteps_per_tile; ++ks) {
          if (!mbar_wait(&full[stage], phase, p.err, kErrTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(smem + stage * p.stage_bytes);
          const uint32_t b = a + p.a_bytes;
          const int steps = (ks % p.nkb == p.nkb - 1) ? p.last_steps : 4;
          for (int s = 0; s < steps; ++s) {
            umma<kInt8>(d, umma_desc_sw128(a + s * 32), umma_desc_sw128(b + s * 32), idesc, accumulate);
            accumulate = 1;
          }
          umma_commit(&empty[stage]);
          if (++stage == p.stages) {
            stage = 0;
            phase ^= 1;
          }
        }
        umma_commit(&tmem_full[acc]);
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const int quarter = warp & 3;  // the TMEM lanes this warp may read
    const int half = (warp - 2) >> 2;  // which half of the tile's channel groups
    const int row = quarter * 32 + lane;
    const bool fast = kInt8 && p.in_zero == 0 && p.out_zero == 0 && p.relu && !p.res && p.c_out == p.cp_out;
    const int groups_all = p.nt / 16, g_lo = half ? (groups_all + 1) / 2 : 0,
              g_hi = half ? groups_all : (groups_all + 1) / 2;
    int iter = 0;
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x, ++iter) {
      const int acc = iter & 1;
      const uint32_t acc_phase = (iter >> 1) & 1;
      if (!mbar_wait(&tmem_full[acc], acc_phase, p.err, kErrTimeoutTmemFull)) break;
      tc_fence_after();
      const int n = t % p.n_tiles, m = t / p.n_tiles;
      const int oy = m / p.m_per_row, ox = (m % p.m_per_row) * 128 + row;
      const bool inside = ox < p.ow;
      const bool valid = inside && p.mask8[(static_cast<long long>(ox) << p.out_shift) >> 3] != 0;
      uint8_t* dst = p.out + (oy + p.out_ph) * p.out_pitch + static_cast<long long>(ox) * p.cp_out * p.ebytes;
      const uint8_t* res = nullptr;
      if (p.res && valid)
        res = p.res + (oy + p.res_ph) * p.res_pitch + static_cast<long long>(ox >> p.res_shift) * p.res_cp * p.ebytes;
      const int c0 = n * p.nt;
      const int cend = min(c0 + p.nt, p.cp_out);
      // 16 channels from r[0..16) to the output at channel cb
      auto store16 = [&](const uint32_t* r, int cb) {
        if (!inside || cb >= cend) return;
        if constexpr (kInt8) {
          alignas(16) uint8_t o[16];
          if (!valid) {
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] = static_cast<uint8_t>(p.out_zero);
          } else if (fast) {
            uint32_t w[4];
#pragma unroll
            for (int i4 = 0; i4 < 4; ++i4) {
              const float4 sc = *reinterpret_cast<const float4*>(s_scale + cb + 4 * i4);
              const float4 bi = *reinterpret_cast<const float4*>(s_bias + cb + 4 * i4);
              const float scs[4] = {sc.x, sc.y, sc.z, sc.w}, bis[4] = {bi.x, bi.y, bi.z, bi.w};
              uint32_t packed = 0;
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const float v = __fadd_rn(__fmul_rn(static_cast<float>(static_cast<int32_t>(r[4 * i4 + k])), scs[k]), bis[k]);
                packed |= cvt_rni_sat_u8(__fmul_rn(v, p.out_inv_scale)) << (8 * k);
              }
              w[i4] = packed;
            }
            *reinterpret_cast<uint4*>(dst + cb) = make_uint4(w[0], w[1], w[2], w[3]);
            return;
          } else {
            alignas(16) uint8_t rb[16];
            if (res) *reinterpret_cast<uint4*>(rb) = *reinterpret_cast<const uint4*>(res + cb);
            const float lo = static_cast<float>(-p.out_zero), hi = static_cast<float>(255 - p.out_zero);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int j = cb + i;
              const int32_t sum = static_cast<int32_t>(r[i]) - p.in_zero * s_colsum[j];
              float v = __fmul_rn(static_cast<float>(sum), s_scale[j]);
              v = __fadd_rn(v, s_bias[j]);
              if (res) v = __fadd_rn(v, __fmul_rn(static_cast<float>(static_cast<int32_t>(rb[i]) - p.res_zero), p.res_scale));
              if (p.relu) v = v > 0.0f ? v : 0.0f;
              float q = __fmul_rn(v, p.out_inv_scale);
              q = q > lo ? q : lo;
              q = q < hi ? q : hi;
              o[i] = static_cast<uint8_t>(__float2int_rn(q) + p.out_zero);
              if (j >= p.c_out) o[i] = static_cast<uint8_t>(p.out_zero);
            }
          }
          *reinterpret_cast<uint4*>(dst + cb) = *reinterpret_cast<const uint4*>(o);
        } else {
          alignas(16) __half o[16];
          if (!valid) {
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] = __float2half_rn(0.0f);
          } else {
            alignas(16) __half rh[16];
            if (res) {
              *reinterpret_cast<uint4*>(rh) = *reinterpret_cast<const uint4*>(res + cb * 2);
              *reinterpret_cast<uint4*>(rh + 8) = *reinterpret_cast<const uint4*>(res + cb * 2 + 16);
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int j = cb + i;
              float v = __fadd_rn(__uint_as_float(r[i]), s_bias[j]);
              if (res) v = __fadd_rn(v, __half2float(rh[i]));
              if (p.relu) v = v > 0.0f ? v : 0.0f;
              o[i] = __float2half_rn(j < p.c_out ? v : 0.0f);
            }
          }
          *reinterpret_cast<uint4*>(dst + cb * 2) = *reinterpret_cast<const uint4*>(o);
          *reinterpret_cast<uint4*>(dst + cb * 2 + 16) = *reinterpret_cast<const uint4*>(o + 8);
        }
      };
      // TMEM read 32 columns at a time, the next load in flight while the current is stored
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * 256);
      if (g_lo < g_hi) {
        uint32_t ra[32], rb[32];
        if (g_lo + 1 < g_hi) tmem_ld32(taddr + g_lo * 16, ra); else tmem_ld16(taddr + g_lo * 16, *reinterpret_cast<uint32_t(*)[16]>(ra));
        tmem_wait_ld();
        tmem_pin(ra);
        for (int g = g_lo; g < g_hi;) {
          const int w = g + 1 < g_hi ? 2 : 1;
          const int gn = g + w;
          if (gn + 1 < g_hi) {
            tmem_ld32(taddr + gn * 16, rb);
          } else if (gn < g_hi) {
            tmem_ld16(taddr + gn * 16, *reinterpret_cast<uint32_t(*)[16]>(rb));
          }
          store16(ra, c0 + g * 16);
          if (w == 2) store16(ra + 16, c0 + g * 16 + 16);
          tmem_wait_ld();
          tmem_pin(rb);
#pragma unroll
          for (int i = 0; i < 32; ++i) ra[i] = rb[i];
          g = gn;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tmem_empty[acc]);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kTmemCols);
}

}  // namespace crec
