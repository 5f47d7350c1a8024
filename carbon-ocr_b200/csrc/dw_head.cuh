// The mixing blocks' depthwise convolution, the recognizer's last layer fused with greedy CTC
// decoding, and the per-line collapse.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "sm100.cuh"

namespace crec {

// ---------------------------------------------------------------- depthwise convolution
//
// Each channel on its own: the int8 sum over taps of (a - zero) * w
// (carbon/src/cpu/kernels.cpp:184-194) or an FP32 sum of FP16 values, then the output stage of
// the dense layers.  The input may be a nearest upsampling read in place: its column u is the
// source's column u >> in_shift (the reference writes the Resize, carbon/src/net/net.cpp:819-851;
// its bytes are a copy of its input, so reading the input is the same).  One thread a pixel
// and 16 channels; gap columns get the zero point.
struct DwParams {
  const uint8_t* in;  // input tensor's first row
  int in_ph, in_cp, in_shift, in_zero;
  long long in_pitch;
  int kh, kw, pt, pl;
  int oh, ow, c, cp;
  const int8_t* w8;  // [taps][cp]
  const float* wf;   // [taps][cp]
  const float* scale;
  const float* bias;
  int out_zero, relu;
  float out_inv_scale;
  uint8_t* out;
  int out_ph;
  long long out_pitch;
  const uint8_t* mask8;
  int out_shift;
};

template <bool kInt8>
__global__ void __launch_bounds__(256) dw_kernel(const __grid_constant__ DwParams p) {
  const int groups = p.cp / 16;
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long total = static_cast<long long>(p.oh) * p.ow * groups;
  if (i >= total) return;
  const int g = static_cast<int>(i % groups);
  const long long pix = i / groups;
  const int ox = static_cast<int>(pix % p.ow), oy = static_cast<int>(pix / p.ow);
  const int eb = kInt8 ? 1 : 2;
  uint8_t* dst = p.out + (oy + p.out_ph) * p.out_pitch + (static_cast<long long>(ox) * p.cp + g * 16) * eb;
  const bool valid = p.mask8[(static_cast<long long>(ox) << p.out_shift) >> 3] != 0;
  const int taps = p.kh * p.kw;
  if constexpr (kInt8) {
    alignas(16) uint8_t o[16];
    if (!valid) {
      for (int u = 0; u < 16; ++u) o[u] = static_cast<uint8_t>(p.out_zero);
    } else {
      int32_t s[16];
      for (int u = 0; u < 16; ++u) s[u] = 0;
      for (int t = 0; t < taps; ++t) {
        const int iy = oy - p.pt + t / p.kw + p.in_ph, ix = (ox - p.pl + t % p.kw) >> p.in_shift;
        alignas(16) uint8_t a[16];
        *reinterpret_cast<uint4*>(a) =
            *reinterpret_cast<const uint4*>(p.in + iy * p.in_pitch + static_cast<long long>(ix) * p.in_cp + g * 16);
        const int8_t* w = p.w8 + t * p.cp + g * 16;
        for (int u = 0; u < 16; ++u) s[u] += (static_cast<int32_t>(a[u]) - p.in_zero) * w[u];
      }
      const float lo = static_cast<float>(-p.out_zero), hi = static_cast<float>(255 - p.out_zero);
      for (int u = 0; u < 16; ++u) {
        const int j = g * 16 + u;
        float v = __fmul_rn(static_cast<float>(s[u]), p.scale[j]);
        v = __fadd_rn(v, p.bias[j]);
        if (p.relu) v = v > 0.0f ? v : 0.0f;
        float q = __fmul_rn(v, p.out_inv_scale);
        q = q > lo ? q : lo;
        q = q < hi ? q : hi;
        o[u] = j < p.c ? static_cast<uint8_t>(__float2int_rn(q) + p.out_zero) : static_cast<uint8_t>(p.out_zero);
      }
    }
    *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(o);
  } else {
    alignas(16) __half o[16];
    if (!valid) {
      for (int u = 0; u < 16; ++u) o[u] = __float2half_rn(0.0f);
    } else {
      float s[16];
      for (int u = 0; u < 16; ++u) s[u] = 0.0f;
      for (int t = 0; t < taps; ++t) {
        const int iy = oy - p.pt + t / p.kw + p.in_ph, ix = (ox - p.pl + t % p.kw) >> p.in_shift;
        alignas(16) __half a[16];
        const uint8_t* src = p.in + iy * p.in_pitch + (static_cast<long long>(ix) * p.in_cp + g * 16) * 2;
        *reinterpret_cast<uint4*>(a) = *reinterpret_cast<const uint4*>(src);
        *reinterpret_cast<uint4*>(a + 8) = *reinterpret_cast<const uint4*>(src + 16);
        const float* w = p.wf + t * p.cp + g * 16;
        for (int u = 0; u < 16; ++u) s[u] = __fmaf_rn(__half2float(a[u]), w[u], s[u]);
      }
      for (int u = 0; u < 16; ++u) {
        const int j = g * 16 + u;
        float v = __fadd_rn(s[u], p.bias[j]);
        if (p.relu) v = v > 0.0f ? v : 0.0f;
        o[u] = __float2half_rn(j < p.c ? v : 0.0f);
      }
    }
    *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(o);
    *reinterpret_cast<uint4*>(dst + 16) = *reinterpret_cast<const uint4*>(o + 8);
  }
}

// ---------------------------------------------------------------- the head fused with CTC's argmax
//
// A tile is 128 frames (columns of the head's input, one row); the 1x1 head runs over the
// classes a chunk at a time (tcgen05.mma, the accumulators double-buffered in TMEM), A loaded
// once a tile, the chunks' weights streamed.  Per frame: the best class, ties to the lower id
// (strictly greater, classes in order), and for a non-blank best its softmax probability.
// INT8: each class's logit requantized to uint8 exactly as the reference stores the head's
// output (the dense epilogue), the codes kept in shared memory, then the probability as
// carbon/src/cpu/kernels.cpp:799-828 computes it: 1 / (the sum in class order of
// exp_neg(table[q_c] - table[q_best])), table[q] = (q - zero) * scale
// (carbon/src/net/net.cpp:1101-1128) -- the same float operations in the same order.
// FP16: the FP32 logits (sum + bias) and an online maximum and sum of exp_neg terms.
// Only each frame's id and probability leave the kernel; the logits are never written.
struct HeadParams {
  CUtensorMap tmap;     // the head's input: (K byte, frame column, row)
  const uint8_t* wimg;  // [chunk][kb][nchunk rows][128 bytes], swizzled
  int nkb, last_steps, classes, nchunk, chunks;  // last_steps: 32-byte K steps in the last K block
  int ow, num_tiles;
  uint32_t a_bytes, b_bytes;  // A: nkb x 16 KB; B: one chunk (nkb blocks)
  const int32_t* colsum;
  const float* scale;
  const float* bias;
  int in_zero, out_zero;
  float out_inv_scale;
  const float* table;  // [256] the u8 logits' values
  const uint8_t* mask8;
  int out_shift;
  int32_t* frame_id;   // [ow]
  float* frame_prob;   // [ow]
  float* logits;       // optional (tests): [ow][classes] each frame's logits as the reference stores them
  int* err;
};

constexpr int kHeadThreads = 192;
constexpr uint32_t kTmemColsHead = 512;

// carbon/src/cpu/kernels.h:216-250 (exp_neg), each multiply and add rounded on its own.
__device__ __forceinline__ float exp_neg_d(float x) {
  x = x > -87.0f ? x : -87.0f;
  const float n = rintf(__fmul_rn(x, 1.44269504088896341f));
  float r = __fsub_rn(x, __fmul_rn(n, 0.693359375f));
  r = __fsub_rn(r, __fmul_rn(n, -2.12194440e-4f));
  float q = 1.9875691500e-4f;
  q = __fadd_rn(__fmul_rn(q, r), 1.3981999507e-3f);
  q = __fadd_rn(__fmul_rn(q, r), 8.3334519073e-3f);
  q = __fadd_rn(__fmul_rn(q, r), 4.1665795894e-2f);
  q = __fadd_rn(__fmul_rn(q, r), 1.6666665459e-1f);
  q = __fadd_rn(__fmul_rn(q, r), 5.0000001201e-1f);
  const float y = __fadd_rn(__fadd_rn(__fmul_rn(q, __fmul_rn(r, r)), r), 1.0f);
  const float s = __int_as_float((static_cast<int32_t>(n) + 127) << 23);
  return __fmul_rn(y, s);
}

template <bool kInt8>
__global__ void __launch_bounds__(kHeadThreads, 1) head_ctc_kernel(const __grid_constant__ HeadParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;                         // A: nkb blocks of [128][128]
  uint8_t* sb = sa + p.a_bytes;               // B: 2 chunk buffers
  uint8_t* codes = sb + 2 * p.b_bytes;        // INT8: [128][classes]
  uint64_t* bars = reinterpret_cast<uint64_t*>(codes + (kInt8 ? 128 * ((p.classes + 15) & ~15) : 0));
  uint64_t* a_full = bars;
  uint64_t* a_empty = bars + 1;
  uint64_t* b_full = bars + 2;      // [2]
  uint64_t* b_empty = bars + 4;     // [2]
  uint64_t* t_full = bars + 6;      // [2]
  uint64_t* t_empty = bars + 8;     // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);
  const int ncls = p.chunks * p.nchunk;
  int32_t* s_colsum = reinterpret_cast<int32_t*>(bars + 16);  // [ncls] per-class constants
  float* s_scale = reinterpret_cast<float*>(s_colsum + ncls);
  float* s_bias = s_scale + ncls;
  int32_t* nb_row = reinterpret_cast<int32_t*>(s_bias + ncls);  // the tile's non-blank frames: row
  int32_t* nb_q = nb_row + 128;                                 // and best code
  int32_t* s_best = nb_q + 128;                                 // each row's best class
  int32_t* nb_count = s_best + 128;                             // [2]: by tile parity
  int32_t* s_abort = nb_count + 2;
  __shared__ float tab[256];
  for (int j = threadIdx.x; j < ncls; j += blockDim.x) {
    s_colsum[j] = p.colsum[j];
    s_scale[j] = p.scale[j];
    s_bias[j] = p.bias[j];
  }
  if (threadIdx.x < 3) nb_count[threadIdx.x] = 0;  // both counters and the abort flag

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  for (int i = threadIdx.x; i < 256; i += blockDim.x) tab[i] = p.table ? p.table[i] : 0.0f;
  if (threadIdx.x == 0) {
    mbar_init(a_full, 1);
    mbar_init(a_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&b_empty[i], 1);
      mbar_init(&t_full[i], 1);
      mbar_init(&t_empty[i], 4);
    }
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemColsHead);
  if (warp == 0 && lane == 0) prefetch_tmap(&p.tmap);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t a_phase = 0, b_phase[2] = {0, 0};
      int bi = 0;
      for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
        if (!mbar_wait(a_empty, a_phase ^ 1, p.err, kErrTimeoutEmpty)) break;
        a_phase ^= 1;
        mbar_expect_tx(a_full, p.a_bytes);
        for (int kb = 0; kb < p.nkb; ++kb) tma_load_3d(sa + kb * 16384, &p.tmap, kb * 128, t * 128, 0, a_full);
        bool ok = true;
        for (int c = 0; c < p.chunks; ++c) {
          if (!mbar_wait(&b_empty[bi], b_phase[bi] ^ 1, p.err, kErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          b_phase[bi] ^= 1;
          mbar_expect_tx(&b_full[bi], p.b_bytes);
          bulk_load(sb + bi * p.b_bytes, p.wimg + static_cast<size_t>(c) * p.b_bytes, p.b_bytes, &b_full[bi]);
          bi ^= 1;
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = kInt8 ? idesc_i8(p.nchunk) : idesc_f16(p.nchunk);
      uint32_t a_phase = 0, b_phase[2] = {0, 0}, t_phase[2] = {0, 0};
      int bi = 0, ti = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
        if (!mbar_wait(a_full, a_phase, p.err, kErrTimeoutFull)) break;
        a_phase ^= 1;
        for (int c = 0; c < p.chunks; ++c) {
          if (!mbar_wait(&t_empty[ti], t_phase[ti] ^ 1, p.err, kErrTimeoutTmemEmpty) ||
              !mbar_wait(&b_full[bi], b_phase[bi], p.err, kErrTimeoutFull)) {
            ok = false;
            break;
          }
          t_phase[ti] ^= 1;
          b_phase[bi] ^= 1;
          tc_fence_after();
          const uint32_t d = tmem_base + static_cast<uint32_t>(ti * 256);
          const uint32_t a0 = smem_u32(sa), b0 = smem_u32(sb + bi * p.b_bytes);
          uint32_t accumulate = 0;
          for (int kb = 0; kb < p.nkb; ++kb) {
            const int steps = kb == p.nkb - 1 ? p.last_steps : 4;
            for (int s = 0; s < steps; ++s) {
              umma<kInt8>(d, umma_desc_sw128(a0 + kb * 16384 + s * 32),
                          umma_desc_sw128(b0 + kb * p.nchunk * 128 + s * 32), idesc, accumulate);
              accumulate = 1;
            }
          }
          umma_commit(&b_empty[bi]);
          umma_commit(&t_full[ti]);
          bi ^= 1;
          ti ^= 1;
        }
        umma_commit(a_empty);
      }
    }
  } else {
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    uint32_t t_phase[2] = {0, 0};
    int ti = 0;
    uint8_t* my = codes + row * ((p.classes + 15) & ~15);
    const float lo = static_cast<float>(-p.out_zero), hi = static_cast<float>(255 - p.out_zero);
    bool ok = true;
    int tile_parity = 0;
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x, tile_parity ^= 1) {
      const int ox = t * 128 + row;
      int best = 0;
      int bestq = -1;
      float bestv = -INFINITY, sum = 0.0f;
      for (int c = 0; c < p.chunks && ok; ++c) {
        if (!mbar_wait(&t_full[ti], t_phase[ti], p.err, kErrTimeoutTmemFull)) {
          ok = false;
          break;
        }
        t_phase[ti] ^= 1;
        tc_fence_after();
        // 16 classes of this chunk, from r[0..16), starting at chunk column cb
        auto take16 = [&](const uint32_t* r, int cb) {
          const int j0 = c * p.nchunk + cb;
          if constexpr (kInt8) {
            alignas(16) uint8_t o[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int j = j0 + i;
              const int32_t s = static_cast<int32_t>(r[i]) - p.in_zero * s_colsum[j];
              float v = __fmul_rn(static_cast<float>(s), s_scale[j]);
              v = __fadd_rn(v, s_bias[j]);
              float q = __fmul_rn(v, p.out_inv_scale);
              q = q > lo ? q : lo;
              q = q < hi ? q : hi;
              const int code = __float2int_rn(q) + p.out_zero;
              o[i] = static_cast<uint8_t>(code);
              if (p.logits && j < p.classes && ox < p.ow) p.logits[static_cast<long long>(ox) * p.classes + j] = tab[code];
              if (j < p.classes && code > bestq) {
                bestq = code;
                best = j;
              }
            }
            if (j0 < ((p.classes + 15) & ~15)) *reinterpret_cast<uint4*>(my + j0) = *reinterpret_cast<const uint4*>(o);
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int j = j0 + i;
              if (j >= p.classes) continue;
              const float v = __fadd_rn(__uint_as_float(r[i]), s_bias[j]);
              if (p.logits && ox < p.ow) p.logits[static_cast<long long>(ox) * p.classes + j] = v;
              if (v > bestv) {
                sum = bestv == -INFINITY ? 1.0f : __fadd_rn(__fmul_rn(sum, exp_neg_d(__fsub_rn(bestv, v))), 1.0f);
                bestv = v;
                best = j;
              } else {
                sum = __fadd_rn(sum, exp_neg_d(__fsub_rn(v, bestv)));
              }
            }
          }
        };
        // TMEM read 32 columns at a time, the next load in flight while the current is taken
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(ti * 256);
        const int groups = p.nchunk / 16;
        uint32_t ra[32], rb[32];
        if (groups >= 2) tmem_ld32(taddr, ra); else tmem_ld16(taddr, *reinterpret_cast<uint32_t(*)[16]>(ra));
        tmem_wait_ld();
        tmem_pin(ra);
        for (int g = 0; g < groups;) {
          const int w = g + 1 < groups ? 2 : 1;
          const int gn = g + w;
          if (gn + 1 < groups) {
            tmem_ld32(taddr + gn * 16, rb);
          } else if (gn < groups) {
            tmem_ld16(taddr + gn * 16, *reinterpret_cast<uint32_t(*)[16]>(rb));
          }
          take16(ra, g * 16);
          if (w == 2) take16(ra + 16, g * 16 + 16);
          tmem_wait_ld();
          tmem_pin(rb);
#pragma unroll
          for (int i = 0; i < 32; ++i) ra[i] = rb[i];
          g = gn;
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&t_empty[ti]);
        ti ^= 1;
      }
      const bool valid = ok && ox < p.ow && p.mask8[(static_cast<long long>(ox) << p.out_shift) >> 3] != 0;
      if constexpr (kInt8) {
        // the class-order sums only for the tile's non-blank frames, gathered into a list so every
        // lane of the warps that run them has one (most frames are blank)
        if (!ok) atomicOr(s_abort, 1);
        s_best[row] = best;
        if (valid && best != 0) {
          const int k = atomicAdd(&nb_count[tile_parity], 1);
          nb_row[k] = row;
          nb_q[k] = bestq;
        } else if (valid) {
          p.frame_id[ox] = 0;
          p.frame_prob[ox] = 0.0f;
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        const int e = threadIdx.x - 64;  // 0..127: this thread's place among the epilogue's
        if (e == 0) nb_count[tile_parity ^ 1] = 0;  // the next tile's counter (its adds follow the next barrier)
        const int listed = nb_count[tile_parity];
        const int stride = (p.classes + 15) & ~15;
        if (!*s_abort) {
          for (int k = e; k < listed; k += 128) {
            const int r = nb_row[k];
            const uint8_t* rowc = codes + r * stride;
            const float top = tab[nb_q[k]];
            float sum = 0.0f;
            for (int j0 = 0; j0 < p.classes; j0 += 16) {
              alignas(16) uint8_t q16[16];
              *reinterpret_cast<uint4*>(q16) = *reinterpret_cast<const uint4*>(rowc + j0);
              float term[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) term[i] = exp_neg_d(__fsub_rn(tab[q16[i]], top));
#pragma unroll
              for (int i = 0; i < 16; ++i)
                if (j0 + i < p.classes) sum = __fadd_rn(sum, term[i]);
            }
            const int fx = t * 128 + r;
            p.frame_id[fx] = s_best[r];
            p.frame_prob[fx] = __fdiv_rn(1.0f, sum);
          }
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (*s_abort) break;
      } else {
        if (!ok) break;
        if (!valid) continue;
        p.frame_id[ox] = best;
        p.frame_prob[ox] = best != 0 ? __fdiv_rn(1.0f, sum) : 0.0f;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kTmemColsHead);
}

// ---------------------------------------------------------------- collapse
//
// carbon/src/lines.cpp:331-355 (ctc_collapse): per line, over its first `length` frames, drop
// blanks and repeats; each character's first frame and the highest probability of its run.
// A line's characters go to its own slots (from its first frame column): at most one a frame.
struct CollapseParams {
  const int32_t* frame_id;
  const float* frame_prob;
  const int* line_frame0;  // [n] the line's first frame column
  const int* length;       // [n] frames read
  int n;
  int32_t* count;  // [n]
  int32_t* ids;    // slots, indexed like the frame columns
  int32_t* frames;
  float* probs;
};

__global__ void collapse_kernel(const __grid_constant__ CollapseParams p) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= p.n) return;
  const int f0 = p.line_frame0[i], len = p.length[i];
  int k = 0, prev = 0;
  for (int t = 0; t < len; ++t) {
    const int id = p.frame_id[f0 + t];
    const float q = p.frame_prob[f0 + t];
    if (id != 0 && id != prev) {
      p.ids[f0 + k] = id;
      p.frames[f0 + k] = t;
      p.probs[f0 + k] = q;
      ++k;
    } else if (id != 0) {
      const float last = p.probs[f0 + k - 1];
      p.probs[f0 + k - 1] = last > q ? last : q;
    }
    prev = id;
  }
  p.count[i] = k;
}

// ---------------------------------------------------------------- packing the decodings
//
// A call's runs each collapse into per-line slots; these pack every line's characters end to
// end, in line order across the runs, so only the characters themselves cross to the host.
// scan_counts_kernel: one CTA; the run's lines' exclusive prefix sum of counts, from the call's
// running total (*total, then advanced by the run's characters).
__global__ void __launch_bounds__(1024) scan_counts_kernel(const int32_t* count, int m, int32_t* counts_out,
                                                           int32_t* offsets_out, long long* total) {
  __shared__ int32_t warp_sums[32];
  __shared__ long long carry;
  if (threadIdx.x == 0) carry = *total;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int base = 0; base < m; base += 1024) {
    const int i = base + static_cast<int>(threadIdx.x);
    const int32_t v = i < m ? count[i] : 0;
    int32_t x = v;  // inclusive scan within the warp
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int32_t w = warp_sums[lane];
      for (int o = 1; o < 32; o <<= 1) {
        const int32_t y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      warp_sums[lane] = w;  // inclusive over warps
    }
    __syncthreads();
    const int32_t before = (warp ? warp_sums[warp - 1] : 0) + x - v;
    if (i < m) {
      counts_out[i] = v;
      offsets_out[i] = static_cast<int32_t>(carry + before);
    }
    __syncthreads();
    if (threadIdx.x == 0) carry += warp_sums[31];
    __syncthreads();
  }
  if (threadIdx.x == 0) *total = carry;
}

// A warp a line: its characters from its slots to the packed arrays at its offset.
__global__ void pack_kernel(const int32_t* ids, const int32_t* frames, const float* probs, const int* line_frame0,
                            const int32_t* counts, const int32_t* offsets, int m, int32_t* out_ids,
                            int32_t* out_frames, float* out_probs) {
  const int warp = static_cast<int>((blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
  if (warp >= m) return;
  const int f0 = line_frame0[warp], k = counts[warp];
  const long long o = offsets[warp];
  for (int j = lane; j < k; j += 32) {
    out_ids[o + j] = ids[f0 + j];
    out_frames[o + j] = frames[f0 + j];
    out_probs[o + j] = probs[f0 + j];
  }
}

}  // namespace crec

