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
// Warp roles (18 warps): 0 TMA producer, 1 MMA issuer (and TMEM owner), 2-17 epilogue: a tile
// is taken by eight warps (warps 2-5 and 10-13 the CTA's even tiles, 6-9 and 14-17 its odd ones),
// each warp the 32 TMEM lanes (pixels) of its quarter (its warp index mod 4) and half of the
// tile's channel groups (2-9 the first half, 10-17 the second).  Up to eight accumulators in TMEM
// (512 columns over the tile's N rounded up to a power of two), so the MMA runs ahead of the
// epilogue.  The epilogue is where an INT8 layer's time goes (requantizing 128 x N outputs costs
// more CUDA-core cycles than the tensor cores' MMAs for K below ~700): the per-channel constants
// in shared memory read four at a time, the line mask of the next tile loaded during this one,
// and the int <-> float conversions done exactly on the FMA pipe (kMagic) wherever the layer's
// sums fit in 22 bits (the host bounds them from the weights), the ReLU folded into the clamp
// (v * inv_scale is monotone, so clamping at 0 is the ReLU).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "sm100.cuh"

namespace crec {

constexpr int kMaxKRows = 12;  // input rows a tile's K runs over

// Row stacking: a tile may compute q_rows output rows at once, N = q_rows x cq (each output
// row's cq channels one after the other), so that a narrow layer's MMAs still fill N (a
// tcgen05.mma of M = 128, K = 32 bytes costs about the same at any N up to 256).  K then runs
// over the (q_rows - 1) * sh + kh input rows the tile's output rows read; the weight image holds
// zeros where an output row does not read an input row.
struct ConvParams {
  CUtensorMap tmap[kMaxKRows];  // one per input row of a tile (3rd coordinate: the tile's row group)
  // a window's last K block when it holds 32 or 64 bytes (tail_bytes; else 128): boxes that wide in
  // the 32- or 64-byte swizzle, the weights' block rows that wide too, so the block's loads carry
  // no padding
  CUtensorMap tmap_tail[kMaxKRows];
  int tail_bytes;
  uint32_t row_bytes;  // without row stacking: an input row's weight blocks, (nkb - 1) * b_bytes + nt * tail_bytes
  const uint8_t* wimg;  // [n tile][ky][kb][nt rows][128 bytes], each block in the 128-byte swizzle
                        // (row stacking: [ky][kb][st_n[ky] rows][128 bytes]); the last kb's rows
                        // tail_bytes wide in their swizzle
  int krows, nkb, last_steps;  // input rows; K blocks of 128 bytes a row; 32-byte K steps in a row's last block
  int q_rows, cq;              // output rows a tile; its channels an output row (cq = nt when q_rows is 1)
  // row stacking: input row i of a tile serves output rows [st_q0[i], st_q0[i] + st_n[i] / cq), so
  // its stages load those rows' weights only (st_n[i] rows of 128 bytes a K block, from byte
  // st_off[i] of wimg) and its MMAs write those rows' accumulator columns; bit i of st_first: input
  // row i is the first an output row reads (its kb 0 starts that row's sum)
  int st_q0[kMaxKRows], st_n[kMaxKRows];
  uint32_t st_off[kMaxKRows];
  uint32_t st_first;
  int cq_inv;                  // ceil(65536 / (cq / 16)): a group g's output row is (g * cq_inv) >> 16 (exact for g < 16)
  int nt, n_tiles;          // output channels a tile (multiple of 16, <= 256), tiles across the channels
  int oh, ow, m_per_row, num_tiles;
  uint32_t nt_magic, mpr_magic;  // div_magic(n_tiles), div_magic(m_per_row): the tile decode without divisions
  int stages;
  uint32_t stage_bytes, a_bytes, b_bytes;
  // epilogue
  uint8_t* out;  // the output tensor's first row (its top border row)
  int out_ph;
  long long out_pitch;  // bytes per output row
  int cp_out, c_out, ebytes;
  const int32_t* off;     // INT8 [cp_out]: kMagicBits - in_zero * colsum (fast), else in_zero * colsum
  const float* scale;     // [cp_out] input scale * weight scale (int8)
  const float* bias;      // [cp_out]
  int out_zero, relu;
  int sat;  // INT8: |v * inv_scale| < 2^21 for every output and no ReLU above a zero point, so the code
           // may be rounded first and clamped to [0, 255] by the saturating pack
  int n_acc;              // TMEM accumulators (a power of two, <= kMaxAcc), each 512 / n_acc columns
  float out_inv_scale;
  const uint8_t* res;  // residual tensor's first row, or null
  int res_ph, res_cp, res_shift, res_zero;
  long long res_pitch;
  float res_scale;
  const uint8_t* mask8;  // one byte per 8 input columns: 1 where a line is
  int out_shift;         // log2 of input columns per output column
  int* err;
  unsigned long long wait_ns;  // every wait's limit (kWaitNs; shorter only for a test's injected timeout)
  int idle_producer;           // test hook: the producer issues nothing, so the waits run out
  // band mode (conv_gemm_kernel<..., kBand = true>): see the comment above the kernel
  int num_bands;               // 128-column bands of the output
  int band_rows;               // input rows a band reads: (oh - 1) * sh + kh
  int kh, kw, sh, pairs, sw;   // kernel, vertical stride, 32-byte channel pairs, horizontal stride
  int plane_px;                // pixel rows a channel plane holds
  int gx0;                     // the first plane row's pixel group, relative to the band's first output column
  int kx_parity[3], kx_off[3]; // per kernel column: its plane's parity and its first row in the plane
  uint32_t slot_bytes;         // a ring slot: one input row, (2 * pairs) x sw planes of plane_px x 16 bytes
  uint32_t load_bytes;         // the bytes a slot's loads bring (the real chunks only)
  int chunks;                  // 16-byte channel chunks of the input (the rest of 2 * pairs stay zero)
  uint32_t w_bytes;            // the resident weight image
  int row0;                    // the input's border rows less the layer's top padding: band row i is map row i + row0
};

static_assert(sizeof(ConvParams) <= 4096, "conv kernel parameters within the classic 4 KB");

constexpr int kConvThreads = 576;
constexpr int kMaxAcc = 8;
constexpr uint32_t kTmemCols = 512;

// The accumulators a layer with tiles of nt channels gets.
__host__ __device__ constexpr int conv_accumulators(int nt) {
  return nt <= 32 ? 8 : nt <= 64 ? 8 : nt <= 128 ? 4 : 2;
}

// Band mode, for narrow layers (few channels, so a tile's K is short and the 128-byte im2col boxes
// would re-read every input row kh x kw times through L2): a CTA takes a band of 128 output
// columns from the first output row to the last.  Each input row the band reads is loaded once,
// into a ring slot of shared memory, as channel planes: for each 16-byte chunk of the channels
// (and, with stride 2, for each pixel parity) the band's pixels one after another, 16 bytes
// each.  That is the tensor cores' K-major layout without swizzle (8-row core matrices of 16
// bytes), so the MMA for kernel tap (ky, kx) and a 32-byte channel pair reads its A operand in
// place: the planes of input row oy * sh + ky, starting kx's row offset in, the next chunk one
// plane further (the descriptor's leading byte offset), the next 8 pixels 128 bytes further
// (its stride byte offset).  The weights stay resident, [ky][kx][pair][N / 8][2][8 rows][16 bytes]
// (the same layout).  The epilogue is the other mode's.
//
// Compile-time forms of a layer, so the epilogue's per-16-channel code carries no run-time
// branches: kRes a residual input, kSat the round-first output stage (p.sat), kStack row stacking
// (p.q_rows > 1), kBand the band mode.
template <bool kInt8, bool kFast, bool kRes, bool kSat, bool kStack, bool kBand>
__global__ void __launch_bounds__(kConvThreads, 1) conv_gemm_kernel(const __grid_constant__ ConvParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-aligned base for the swizzled stages (band mode: the resident weights, then the ring)
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t data_bytes = kBand ? p.w_bytes + p.stages * p.slot_bytes : p.stages * p.stage_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + data_bytes);
  uint64_t* empty = full + p.stages;
  uint64_t* tmem_full = empty + p.stages;      // [kMaxAcc]
  uint64_t* tmem_empty = tmem_full + kMaxAcc;  // [kMaxAcc]
  uint64_t* w_full = tmem_empty + kMaxAcc;     // band mode: the resident weights (16 bytes kept, so
                                               // the per-channel tables below stay 16-byte aligned)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(w_full + 2);
  int32_t* s_off = reinterpret_cast<int32_t*>(tmem_slot + 4);  // [cp_out] per-channel constants
  float* s_scale = reinterpret_cast<float*>(s_off + p.cp_out);
  float* s_bias = s_scale + p.cp_out;
  for (int j = threadIdx.x; j < p.cp_out; j += blockDim.x) {
    s_off[j] = kInt8 ? p.off[j] : 0;
    s_scale[j] = p.scale[j];
    s_bias[j] = p.bias[j];
  }

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < kMaxAcc; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], 8);  // the eight warps of the half that takes the tile
    }
    mbar_init(w_full, 1);
    fence_mbar_init();
  }
  if constexpr (kBand) {
    // the ring's planes past the input's chunks (a channel pair's missing half) hold zeros: the
    // loads never write them, and zero times a zero weight is zero (float16 too)
    const int planes = 2 * p.pairs * p.sw, real = p.chunks * p.sw;
    const uint32_t plane_bytes = static_cast<uint32_t>(p.plane_px) * 16;
    for (int s = 0; s < p.stages; ++s)
      for (uint32_t i = threadIdx.x * 16; i < (planes - real) * plane_bytes; i += blockDim.x * 16)
        *reinterpret_cast<uint4*>(smem + p.w_bytes + s * p.slot_bytes + real * plane_bytes + i) = make_uint4(0, 0, 0, 0);
    fence_proxy_async_smem();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  if (warp == 0 && lane == 0) {
    for (int k = 0; k < p.krows; ++k) prefetch_tmap(&p.tmap[k]);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int ksteps_per_tile = p.krows * p.nkb;
  const uint32_t acc_cols = kTmemCols / static_cast<uint32_t>(p.n_acc);

  if (kBand && warp == 0) {
    // ---------------------------------------------------------------- band producer
    // the weights once, then each band's input rows into the ring, in order
    const bool leader = elect_one();
    if (leader) {
      mbar_expect_tx(w_full, p.w_bytes);
      for (uint32_t off = 0; off < p.w_bytes; off += 32768)
        bulk_load(smem + off, p.wimg + off, min(32768u, p.w_bytes - off), w_full);
    }
    __syncwarp();
    uint32_t g = 0;  // rows loaded so far
    bool ok = p.idle_producer == 0;
    for (int band = blockIdx.x; band < p.num_bands && ok; band += gridDim.x) {
      const int c = band * 128 + p.gx0;
      for (int i = 0; i < p.band_rows; ++i, ++g) {
        const int slot = static_cast<int>(g % static_cast<uint32_t>(p.stages));
        const uint32_t phase = (g / static_cast<uint32_t>(p.stages)) & 1;
        if (!mbar_wait_warp(&empty[slot], phase ^ 1, p.err, kErrTimeoutEmpty, p.wait_ns)) {
          ok = false;
          break;
        }
        if (leader) {
          uint8_t* dst = smem + p.w_bytes + slot * p.slot_bytes;
          mbar_expect_tx(&full[slot], p.load_bytes);
          for (int j = 0; j < p.chunks; ++j)
            for (int par = 0; par < p.sw; ++par)
              tma_load_4d(dst + (j * p.sw + par) * p.plane_px * 16, &p.tmap[0], 16 * j, par, c, i + p.row0, &full[slot]);
        }
        __syncwarp();
      }
    }
  } else if (kBand && warp == 1) {
    // ---------------------------------------------------------------- band MMA issuer
    const bool leader = elect_one();
    const uint32_t tmem = __shfl_sync(0xffffffffu, tmem_base, 0);
    const uint32_t ring = smem_u32(smem) + p.w_bytes, plane_bytes = static_cast<uint32_t>(p.plane_px) * 16;
    const uint32_t lbo = static_cast<uint32_t>(p.sw) * plane_bytes;  // the next 16-byte chunk, same parity
    const uint32_t w_step = static_cast<uint32_t>(p.cq) * 32;
    const uint64_t a_desc0 = umma_desc_none(ring, lbo, 128), b_desc0 = umma_desc_none(smem_u32(smem), 128, 256);
    bool ok = mbar_wait_warp(w_full, 0, p.err, kErrTimeoutFull, p.wait_ns);
    tc_fence_after();
    uint32_t g = 0;  // the ring counter of the band's first row
    int s = 0;       // this CTA's tile sequence
    const int groups = p.oh / p.q_rows;
    const uint32_t idesc_row = kInt8 ? idesc_i8(p.cq) : idesc_f16(p.cq);  // one output row's channels
    for (int band = blockIdx.x; band < p.num_bands && ok; band += gridDim.x) {
      for (int grp = 0; grp < groups && ok; ++grp, ++s) {
        const int acc = s & (p.n_acc - 1);
        if (!mbar_wait_warp(&tmem_empty[acc], ((s / p.n_acc) & 1) ^ 1, p.err, kErrTimeoutTmemEmpty, p.wait_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // output row oy = grp * q_rows + q of the tile into accumulator columns [q * cq, (q + 1) * cq)
        for (int q = 0; q < p.q_rows && ok; ++q) {
          const int oy = grp * p.q_rows + q;
          const uint32_t d = tmem + static_cast<uint32_t>(acc) * acc_cols + static_cast<uint32_t>(q * p.cq);
          uint32_t accumulate = 0;
          for (int ky = 0; ky < p.kh && ok; ++ky) {
            const uint32_t r = g + static_cast<uint32_t>(oy * p.sh + ky);
            const uint32_t slot = r % static_cast<uint32_t>(p.stages);
            if (!mbar_wait_warp(&full[slot], (r / static_cast<uint32_t>(p.stages)) & 1, p.err, kErrTimeoutFull, p.wait_ns)) {
              ok = false;
              break;
            }
            tc_fence_after();
            // every lane computes the descriptors (warp-uniform values); one lane issues.  A tap's
            // descriptors differ from the row's (and the weights' first) only in the start address
            // field (address >> 4, no carry: shared memory is below 256 KB)
            const uint64_t row_desc = a_desc0 + ((slot * p.slot_bytes) >> 4);
            uint64_t bd = b_desc0 + static_cast<uint64_t>((ky * p.kw * p.pairs * w_step) >> 4);
            for (int kx = 0; kx < p.kw; ++kx) {
              uint64_t ad = row_desc + ((static_cast<uint32_t>(p.kx_parity[kx]) * plane_bytes + static_cast<uint32_t>(p.kx_off[kx]) * 16) >> 4);
              for (int pr = 0; pr < p.pairs; ++pr) {
                if (leader) umma<kInt8>(d, ad, bd, idesc_row, accumulate);
                accumulate = 1;
                ad += (2 * lbo) >> 4;
                bd += w_step >> 4;
              }
            }
            __syncwarp();
          }
        }
        if (!ok) break;
        if (leader) {
          umma_commit(&tmem_full[acc]);
          // the rows no later tile of the band reads go back to the producer
          const int first = grp * p.q_rows * p.sh, last = grp + 1 == groups ? p.band_rows : (grp + 1) * p.q_rows * p.sh;
          for (int i = first; i < last; ++i) umma_commit(&empty[(g + static_cast<uint32_t>(i)) % static_cast<uint32_t>(p.stages)]);
        }
        __syncwarp();
      }
      g += static_cast<uint32_t>(p.band_rows);
    }
  } else if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    // The whole warp runs the loop (its counters, coordinates and addresses warp-uniform), one
    // elected lane issues the copies.
    const bool leader = elect_one();
    int stage = 0;
    uint32_t phase = 0;
    bool ok = p.idle_producer == 0;
    for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
      const int m = fast_div(t, p.n_tiles, p.nt_magic), n = t - m * p.n_tiles;
      const int oy = fast_div(m, p.m_per_row, p.mpr_magic), ox0 = (m - oy * p.m_per_row) * 128;
      for (int ky = 0; ky < p.krows && ok; ++ky) {
        for (int kb = 0; kb < p.nkb; ++kb) {
          if (!mbar_wait_warp(&empty[stage], phase ^ 1, p.err, kErrTimeoutEmpty, p.wait_ns)) {
            ok = false;
            break;
          }
          if (leader) {
            uint8_t* a = smem + stage * p.stage_bytes;
            uint8_t* b = a + p.a_bytes;
            const bool tail = kb == p.nkb - 1 && p.tail_bytes < 128;
            const uint32_t pitch = tail ? static_cast<uint32_t>(p.tail_bytes) : 128u;  // a block row's bytes
            const uint32_t rows = kStack ? static_cast<uint32_t>(p.st_n[ky]) : static_cast<uint32_t>(p.nt);
            const uint32_t ab = 128u * pitch, bb = rows * pitch;
            mbar_expect_tx(&full[stage], ab + bb);
            tma_load_3d(a, tail ? &p.tmap_tail[ky] : &p.tmap[ky], kb * 128, ox0, oy, &full[stage]);
            const uint8_t* w = kStack ? p.wimg + p.st_off[ky] + static_cast<size_t>(kb) * rows * 128u
                                      : p.wimg + static_cast<size_t>(n * p.krows + ky) * p.row_bytes +
                                            static_cast<size_t>(kb) * p.b_bytes;
            bulk_load(b, w, bb, &full[stage]);
          }
          __syncwarp();
          if (++stage == p.stages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    // As the producer: the warp runs the loop, so the descriptors, the accumulator address and
    // the accumulate flag the MMAs take are warp-uniform; one elected lane issues the MMAs and
    // their commits (a commit tracks the MMAs of the lane that issues it).
    const bool leader = elect_one();
    const uint32_t tmem = __shfl_sync(0xffffffffu, tmem_base, 0);
    const uint32_t idesc = kInt8 ? idesc_i8(p.nt) : idesc_f16(p.nt);
    // the stages' descriptors differ only in the start address (bits 0..13, address >> 4): a
    // K step of 32 bytes adds 2, a stage stage_bytes >> 4
    const uint64_t a_desc0 = umma_desc_sw128(smem_u32(smem)), b_desc0 = umma_desc_sw128(smem_u32(smem) + p.a_bytes);
    const bool narrow = p.tail_bytes < 128;
    const uint32_t tail_row = narrow ? static_cast<uint32_t>(p.tail_bytes) : 128u;
    const uint64_t a_tail0 = narrow ? umma_desc_narrow(smem_u32(smem), tail_row) : a_desc0;
    const uint64_t b_tail0 = narrow ? umma_desc_narrow(smem_u32(smem) + p.a_bytes, tail_row) : b_desc0;
    const uint32_t stage_step = p.stage_bytes >> 4;
    int stage = 0;
    uint32_t phase = 0;
    int iter = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x, ++iter) {
      const int acc = iter & (p.n_acc - 1);
      const uint32_t acc_phase = (iter / p.n_acc) & 1;
      if (!mbar_wait_warp(&tmem_empty[acc], acc_phase ^ 1, p.err, kErrTimeoutTmemEmpty, p.wait_ns)) break;
      tc_fence_after();
      const uint32_t d = tmem + static_cast<uint32_t>(acc) * acc_cols;
      uint32_t accumulate = 0;
      int kb = 0, ky = 0;
      for (int ks = 0; ks < ksteps_per_tile; ++ks) {
        if (!mbar_wait_warp(&full[stage], phase, p.err, kErrTimeoutFull, p.wait_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int kb_now = kb, ky_now = ky;
        const bool tail = narrow && kb_now == p.nkb - 1;
        const uint64_t ad = (tail ? a_tail0 : a_desc0) + static_cast<uint64_t>(stage) * stage_step;
        const uint64_t bd = (tail ? b_tail0 : b_desc0) + static_cast<uint64_t>(stage) * stage_step;
        const int steps = ++kb == p.nkb ? p.last_steps : 4;
        if (kb == p.nkb) {
          kb = 0;
          ++ky;
        }
        if constexpr (kStack) {
          // the output rows this input row serves: one MMA over their columns, except at the first
          // K step of the row that starts here, where that row's MMA begins its sum (accumulate 0)
          // beside the earlier rows' (accumulate 1); B's rows are the served rows' in order, so the
          // new row's are the last cq (whole 8-row groups: the swizzle is unchanged)
          const int nq = p.st_n[ky_now];
          const uint32_t dq = d + static_cast<uint32_t>(p.st_q0[ky_now] * p.cq);
          const uint32_t id = kInt8 ? idesc_i8(nq) : idesc_f16(nq);
          const bool starts = kb_now == 0 && ((p.st_first >> ky_now) & 1u);
          const int nold = nq - p.cq;
          if (leader) {
#pragma unroll
            for (int s = 0; s < 4; ++s) {
              if (s >= steps) continue;
              if (s == 0 && starts) {
                if (nold > 0) umma<kInt8>(dq, ad, bd, kInt8 ? idesc_i8(nold) : idesc_f16(nold), 1u);
                const uint32_t pitch = tail ? tail_row : 128u;
                umma<kInt8>(dq + static_cast<uint32_t>(nold), ad, bd + static_cast<uint64_t>((static_cast<uint32_t>(nold) * pitch) >> 4),
                            kInt8 ? idesc_i8(p.cq) : idesc_f16(p.cq), 0u);
              } else {
                umma<kInt8>(dq, ad + 2 * s, bd + 2 * s, id, 1u);
              }
            }
            umma_commit(&empty[stage]);
          }
        } else if (leader) {
#pragma unroll
          for (int s = 0; s < 4; ++s)
            if (s < steps) umma<kInt8>(d, ad + 2 * s, bd + 2 * s, idesc, accumulate | static_cast<uint32_t>(s));
          umma_commit(&empty[stage]);
        }
        __syncwarp();
        accumulate = 1;
        if (++stage == p.stages) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (leader) umma_commit(&tmem_full[acc]);
      __syncwarp();
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const int quarter = warp & 3;           // the TMEM lanes this warp may read
    const int half = ((warp - 2) >> 2) & 1;  // the CTA's even (0) or odd (1) tiles
    const int part = (warp - 2) >> 3;       // the first (0) or second (1) part of a tile's channel groups
    const int row = quarter * 32 + lane;
    const int groups = p.nt / 16;
    // the part's 16-channel groups: [g0, g1) (the first part an even count: whole 32-column loads)
    const int gsplit = ((groups + 3) >> 2) << 1;
    const int g0 = part ? min(gsplit, groups) : 0, g1 = part ? groups : min(gsplit, groups);
    const float lo = p.relu ? 0.0f : static_cast<float>(-p.out_zero), hi = static_cast<float>(255 - p.out_zero);
    const int32_t zc = p.out_zero - kMagicBits, rzc = kMagicBits - p.res_zero;
    const uint32_t zb = static_cast<uint32_t>(p.out_zero) * 0x01010101u;
    // INT8 without row stacking and a pixel's channels a multiple of 32 bytes: a thread's two groups
    // of a TMEM read (an even group first) are 32 aligned contiguous bytes, stored at once
    const bool pair32 = !kStack && (p.cp_out * p.ebytes) % 32 == 0;
    // this CTA's tile s: its first output row, its first output column, its channel tile (false
    // past the last one).  Tiles go round the CTAs (tile blockIdx.x + s * gridDim.x), or in band
    // mode band by band, each band's output rows in order
    auto tile_of = [&](int s, int& oy, int& ox0, int& n) -> bool {
      if constexpr (kBand) {
        const int groups = p.oh / p.q_rows;
        const int band = blockIdx.x + (s / groups) * gridDim.x;
        if (band >= p.num_bands) return false;
        oy = (s % groups) * p.q_rows;
        ox0 = band * 128;
        n = 0;
      } else {
        const int t = blockIdx.x + s * gridDim.x;
        if (t >= p.num_tiles) return false;
        const int m = fast_div(t, p.n_tiles, p.nt_magic);
        n = t - m * p.n_tiles;
        const int mr = fast_div(m, p.m_per_row, p.mpr_magic);
        oy = mr * p.q_rows;
        ox0 = (m - mr * p.m_per_row) * 128;
      }
      return true;
    };
    // the line mask byte of this thread's pixel in tile s (0 past the output's width)
    auto mask_of = [&](int s) -> int {
      int oy, ox0, n;
      if (!tile_of(s, oy, ox0, n)) return 0;
      const int ox = ox0 + row;
      return ox < p.ow ? __ldg(p.mask8 + ((static_cast<long long>(ox) << p.out_shift) >> 3)) : 0;
    };
    int iter = half;
    int mk = mask_of(iter);
    int oy, ox0, n;
    for (; tile_of(iter, oy, ox0, n); iter += 2) {
      const int mk_next = mask_of(iter + 2);  // in flight during this tile
      const int acc = iter & (p.n_acc - 1);
      const uint32_t acc_phase = (iter / p.n_acc) & 1;
      if (!mbar_wait(&tmem_full[acc], acc_phase, p.err, kErrTimeoutTmemFull, p.wait_ns)) break;
      tc_fence_after();
      const int ox = ox0 + row;
      const bool inside = ox < p.ow;
      const bool valid = inside && mk != 0;
      mk = mk_next;
      uint8_t* dst0 = p.out + (oy + p.out_ph) * p.out_pitch + static_cast<long long>(ox) * p.cp_out * p.ebytes;
      const uint8_t* res = nullptr;
      if (kRes && valid)
        res = p.res + (oy + p.res_ph) * p.res_pitch + static_cast<long long>(ox >> p.res_shift) * p.res_cp * p.ebytes;
      const int c0 = n * p.nt;
      // INT8: the codes of 16 of the tile's columns from r[0..16), output channels cb on
      auto code16 = [&](const uint32_t* r, int cb) -> uint4 {
          uint4 o;
          if (!valid) {
            o = make_uint4(zb, zb, zb, zb);
          } else if constexpr (kFast) {
            // the output stage; where the layer's bound allows, rounded before the clamp and the
            // clamp done by the saturating byte pack (clamp and round-to-integer commute for
            // integer bounds)
            int32_t code[16];
            uint4 rv = make_uint4(0, 0, 0, 0);
            if constexpr (kRes) rv = *reinterpret_cast<const uint4*>(res + cb);
            const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const int4 o4 = *reinterpret_cast<const int4*>(s_off + cb + 4 * k);
              const float4 s4 = *reinterpret_cast<const float4*>(s_scale + cb + 4 * k);
              const float4 b4 = *reinterpret_cast<const float4*>(s_bias + cb + 4 * k);
              const int32_t oo[4] = {o4.x, o4.y, o4.z, o4.w};
              const float ss[4] = {s4.x, s4.y, s4.z, s4.w}, bb[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
              for (int u = 0; u < 4; u += 2) {
                // two channels at a time on the packed FP32 pipe (the same roundings as scalar)
                const int32_t a0 = static_cast<int32_t>(r[4 * k + u]), a1 = static_cast<int32_t>(r[4 * k + u + 1]);
                float2 v = fadd2_rn(fmul_pair_rn(magic_to_float2(a0 + oo[u], a1 + oo[u + 1]), make_float2(ss[u], ss[u + 1])),
                                    make_float2(bb[u], bb[u + 1]));
                if constexpr (kRes) {
                  const int32_t r0 = static_cast<int32_t>((rw[k] >> (8 * u)) & 0xffu);
                  const int32_t r1 = static_cast<int32_t>((rw[k] >> (8 * u + 8)) & 0xffu);
                  v = fadd2_rn(v, fmul_pair_rn(magic_to_float2(r0 + rzc, r1 + rzc), make_float2(p.res_scale, p.res_scale)));
                }
                float2 q = fmul_pair_rn(v, make_float2(p.out_inv_scale, p.out_inv_scale));
                if constexpr (!kSat) {
                  q.x = fminf(fmaxf(q.x, lo), hi);
                  q.y = fminf(fmaxf(q.y, lo), hi);
                }
                int32_t t0, t1;
                magic_rint_bits2(q, t0, t1);
                code[4 * k + u] = t0 + zc;
                code[4 * k + u + 1] = t1 + zc;
              }
            }
            if (cb + 16 > p.c_out) {
#pragma unroll
              for (int i = 0; i < 16; ++i)
                if (cb + i >= p.c_out) code[i] = p.out_zero;
            }
            o = make_uint4(pack_sat_u8x4(code), pack_sat_u8x4(code + 4), pack_sat_u8x4(code + 8), pack_sat_u8x4(code + 12));
          } else {
            int32_t code[16];
            uint4 rv = make_uint4(0, 0, 0, 0);
            if constexpr (kRes) rv = *reinterpret_cast<const uint4*>(res + cb);
            const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const int4 o4 = *reinterpret_cast<const int4*>(s_off + cb + 4 * k);
              const float4 s4 = *reinterpret_cast<const float4*>(s_scale + cb + 4 * k);
              const float4 b4 = *reinterpret_cast<const float4*>(s_bias + cb + 4 * k);
              const int32_t oo[4] = {o4.x, o4.y, o4.z, o4.w};
              const float ss[4] = {s4.x, s4.y, s4.z, s4.w}, bb[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
              for (int u = 0; u < 4; u += 2) {
                // sums past 2^22: float(s) exactly (round to nearest even) by the split conversion,
                // two channels at a time on the packed FP32 pipe
                const int32_t a0 = static_cast<int32_t>(r[4 * k + u]), a1 = static_cast<int32_t>(r[4 * k + u + 1]);
                float2 v = fadd2_rn(fmul_pair_rn(exact_i2f2(a0 - oo[u], a1 - oo[u + 1]), make_float2(ss[u], ss[u + 1])),
                                    make_float2(bb[u], bb[u + 1]));
                if constexpr (kRes) {
                  const int32_t r0 = static_cast<int32_t>((rw[k] >> (8 * u)) & 0xffu);
                  const int32_t r1 = static_cast<int32_t>((rw[k] >> (8 * u + 8)) & 0xffu);
                  v = fadd2_rn(v, fmul_pair_rn(magic_to_float2(r0 + rzc, r1 + rzc), make_float2(p.res_scale, p.res_scale)));
                }
                float2 q = fmul_pair_rn(v, make_float2(p.out_inv_scale, p.out_inv_scale));
                if constexpr (!kSat) {
                  q.x = fminf(fmaxf(q.x, lo), hi);
                  q.y = fminf(fmaxf(q.y, lo), hi);
                }
                int32_t t0, t1;
                magic_rint_bits2(q, t0, t1);
                code[4 * k + u] = t0 + zc;
                code[4 * k + u + 1] = t1 + zc;
              }
            }
            if (cb + 16 > p.c_out) {
#pragma unroll
              for (int i = 0; i < 16; ++i)
                if (cb + i >= p.c_out) code[i] = p.out_zero;
            }
            o = make_uint4(pack_sat_u8x4(code), pack_sat_u8x4(code + 4), pack_sat_u8x4(code + 8), pack_sat_u8x4(code + 12));
          }
          return o;
      };
      // 16 of the tile's columns from r[0..16), starting at tile column tc: output row oy + q, channel cb
      auto store16 = [&](const uint32_t* r, int tc) {
        const int q = kStack ? ((tc >> 4) * p.cq_inv) >> 16 : 0;
        const int cb = c0 + tc - q * p.cq;
        if (!inside || cb >= p.cp_out || oy + q >= p.oh) return;
        uint8_t* dst = dst0 + q * p.out_pitch;
        if constexpr (kInt8) {
          *reinterpret_cast<uint4*>(dst + cb) = code16(r, cb);
        } else {
          alignas(16) __half o[16];
          if (!valid) {
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] = __float2half_rn(0.0f);
          } else {
            alignas(16) __half rh[16];
            if constexpr (kRes) {
              *reinterpret_cast<uint4*>(rh) = *reinterpret_cast<const uint4*>(res + cb * 2);
              *reinterpret_cast<uint4*>(rh + 8) = *reinterpret_cast<const uint4*>(res + cb * 2 + 16);
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int j = cb + i;
              float v = __fadd_rn(__uint_as_float(r[i]), s_bias[j]);
              if constexpr (kRes) v = __fadd_rn(v, __half2float(rh[i]));
              if (p.relu) v = v > 0.0f ? v : 0.0f;
              o[i] = __float2half_rn(j < p.c_out ? v : 0.0f);
            }
          }
          // one 32-byte store: a pixel's channel pitch and cb * 2 are multiples of 32 bytes
          st_global_v8(dst + cb * 2, *reinterpret_cast<const uint4*>(o), *reinterpret_cast<const uint4*>(o + 8));
        }
      };
      // TMEM read 32 columns at a time (the other warps on the SM hide the loads' latency); the
      // accumulator goes back to the MMA as soon as the part's last load has completed (a warp
      // without groups still waits for the accumulator, so that its arrival counts for this use)
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc) * acc_cols;
      auto release = [&]() {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tmem_empty[acc]);
      };
      if (g0 >= g1) release();
      uint32_t ra[32];
      for (int g = g0; g < g1; g += 2) {
        const int w = g + 1 < g1 ? 2 : 1;
        if (w == 2) tmem_ld32(taddr + g * 16, ra);
        else tmem_ld16(taddr + g * 16, *reinterpret_cast<uint32_t(*)[16]>(ra));
        tmem_wait_ld();
        tmem_pin(ra);
        if (g + w >= g1) release();
        if (kInt8 && pair32 && w == 2 && inside && c0 + g * 16 + 32 <= p.cp_out) {
          // two groups of one pixel, 32 contiguous bytes: one full-sector store
          const int cb = c0 + g * 16;
          st_global_v8(dst0 + cb, code16(ra, cb), code16(ra + 16, cb + 16));
        } else {
          store16(ra, g * 16);
          if (w == 2) store16(ra + 16, g * 16 + 16);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kTmemCols);
}

}  // namespace crec
