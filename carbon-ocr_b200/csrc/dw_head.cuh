// The mixing blocks' depthwise convolution, the recognizer's last layer fused with greedy CTC
// decoding, and the per-line collapse.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "crop_stem.cuh"  // dp4a_us
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
  int sat;  // INT8 row kernel: |v * inv_scale| < 2^21 always (round first, clamp while packing)
  float out_inv_scale;
  uint8_t* out;
  int out_ph;
  long long out_pitch;
  const uint8_t* mask8;
  int out_shift;
  // the row kernel (INT8, one kernel row, kw <= 12); channel c = 16 g + 4 q + u of G = cp / 16
  // groups sits at ((slot * 4 + q) * G + g) * 4 + u, so that the 16 groups of a warp's
  // threads read 16 consecutive 16-byte words
  const uint32_t* wt;   // [3 slots]: channel c's taps 4j .. 4j+3 in slot j (zeros past kw)
  const uint32_t* dwc;  // [3 slots]: kMagicBits - in_zero * (the channel's weight sum), scale, bias (bits)
  uint32_t g_magic;     // div_magic(cp / 16): an item's pixel without a division (item * groups < 2^32)
};

// The row kernel's interleaved index of channel c (of cp) in slot `slot`.
__host__ __device__ inline int dw_row_index(int slot, int c, int cp) {
  const int g = c >> 4, q = (c >> 2) & 3, u = c & 3;
  return ((slot * 4 + q) * (cp >> 4) + g) * 4 + u;
}

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

// The INT8 depthwise convolution of one kernel row (1 x kw, kw <= 12), a CTA a tile of
// kDwTile output pixels of one row and all channels.  The input columns the tile reads are
// staged in shared memory with 16-byte loads; a thread takes a (pixel, 16 channels) item: the
// taps' bytes, four taps by four channels at a time, are transposed with byte permutes so that
// each channel's four taps are one word, and dp4a sums them against the channel's weights
// (stored tap-transposed).  The sum is the reference's integer sum of (a - zero) * w (through
// the weights' sum), |sum| <= 12 * 255 * 128 < 2^22, so the output stage converts exactly with
// kMagic.
constexpr int kDwTile = 64;

__host__ __device__ inline int dw_row_cols(int kw, int in_shift) { return ((kDwTile - 1 + kw - 1) >> in_shift) + 2; }

template <bool kSat>
__global__ void __launch_bounds__(256) dw_row_kernel(const __grid_constant__ DwParams p) {
  extern __shared__ __align__(16) uint8_t sm[];
  const int cp = p.cp, G = cp >> 4;
  const int tiles_per_row = (p.ow + kDwTile - 1) / kDwTile;
  const int oy = blockIdx.x / tiles_per_row, ox0 = (blockIdx.x - oy * tiles_per_row) * kDwTile;
  const int sh = p.in_shift;
  const int pc0 = (ox0 - p.pl) >> sh;  // the first input column the tile reads (arithmetic shift: floor)
  const int ncols = dw_row_cols(p.kw, sh);
  uint8_t* sin = sm;  // [ncols][cp]
  uint32_t* swt = reinterpret_cast<uint32_t*>(sm + ((ncols * cp + 15) & ~15));  // [3 slots], interleaved
  uint32_t* sc = swt + 3 * cp;                                                  // [3 slots], interleaved
  {
    const uint8_t* src = p.in + static_cast<long long>(oy - p.pt + p.in_ph) * p.in_pitch + static_cast<long long>(pc0) * cp;
    const int n16 = ncols * cp / 16;
    for (int i = threadIdx.x; i < n16; i += blockDim.x)
      reinterpret_cast<uint4*>(sin)[i] = __ldg(reinterpret_cast<const uint4*>(src) + i);
    for (int i = threadIdx.x; i < 3 * cp; i += blockDim.x) {
      swt[i] = p.wt[i];
      sc[i] = p.dwc[i];
    }
  }
  __syncthreads();
  const float lo = p.relu ? 0.0f : static_cast<float>(-p.out_zero), hi = static_cast<float>(255 - p.out_zero);
  const int32_t zc = p.out_zero - kMagicBits;
  const uint32_t zb = static_cast<uint32_t>(p.out_zero) * 0x01010101u;
  for (int it = threadIdx.x; it < kDwTile * G; it += blockDim.x) {
    const int px = fast_div(it, G, p.g_magic), g = it - px * G;
    const int ox = ox0 + px;
    if (ox >= p.ow) continue;
    uint8_t* dst = p.out + static_cast<long long>(oy + p.out_ph) * p.out_pitch + static_cast<long long>(ox) * cp + g * 16;
    if (p.mask8[(static_cast<long long>(ox) << p.out_shift) >> 3] == 0) {
      *reinterpret_cast<uint4*>(dst) = make_uint4(zb, zb, zb, zb);
      continue;
    }
    const int c0 = g * 16;
    const uint4* sc4 = reinterpret_cast<const uint4*>(sc);  // slot s, quad k: sc4[(s * 4 + k) * G + g]
    int32_t acc[16];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int4 o4 = *reinterpret_cast<const int4*>(sc4 + k * G + g);
      acc[4 * k] = o4.x;
      acc[4 * k + 1] = o4.y;
      acc[4 * k + 2] = o4.z;
      acc[4 * k + 3] = o4.w;
    }
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      if (4 * j >= p.kw) break;
      uint32_t a[4][4];
#pragma unroll
      for (int tt = 0; tt < 4; ++tt) {
        const int t = 4 * j + tt;
        if (t < p.kw) {
          const int col = ((ox - p.pl + t) >> sh) - pc0;
          const uint4 v = *reinterpret_cast<const uint4*>(sin + col * cp + c0);
          a[tt][0] = v.x;
          a[tt][1] = v.y;
          a[tt][2] = v.z;
          a[tt][3] = v.w;
        } else {
          a[tt][0] = a[tt][1] = a[tt][2] = a[tt][3] = 0u;
        }
      }
      const uint4* w4 = reinterpret_cast<const uint4*>(swt);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 wq = w4[(j * 4 + q) * G + g];
        const uint32_t x01l = __byte_perm(a[0][q], a[1][q], 0x5140), x01h = __byte_perm(a[0][q], a[1][q], 0x7362);
        const uint32_t x23l = __byte_perm(a[2][q], a[3][q], 0x5140), x23h = __byte_perm(a[2][q], a[3][q], 0x7362);
        acc[4 * q] = dp4a_us(__byte_perm(x01l, x23l, 0x5410), wq.x, acc[4 * q]);
        acc[4 * q + 1] = dp4a_us(__byte_perm(x01l, x23l, 0x7632), wq.y, acc[4 * q + 1]);
        acc[4 * q + 2] = dp4a_us(__byte_perm(x01h, x23h, 0x5410), wq.z, acc[4 * q + 2]);
        acc[4 * q + 3] = dp4a_us(__byte_perm(x01h, x23h, 0x7632), wq.w, acc[4 * q + 3]);
      }
    }
    uint32_t wv[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float4 s4 = *reinterpret_cast<const float4*>(sc4 + (4 + k) * G + g);
      const float4 b4 = *reinterpret_cast<const float4*>(sc4 + (8 + k) * G + g);
      const float ss[4] = {s4.x, s4.y, s4.z, s4.w}, bb[4] = {b4.x, b4.y, b4.z, b4.w};
      int32_t code[4];
#pragma unroll
      for (int u = 0; u < 4; u += 2) {  // two channels at a time on the packed FP32 pipe
        float2 q = out_stage2(acc[4 * k + u], acc[4 * k + u + 1], make_float2(ss[u], ss[u + 1]),
                              make_float2(bb[u], bb[u + 1]), p.out_inv_scale);
        if constexpr (!kSat) {  // with kSat the clamp is the saturating pack (rounding first is exact there)
          q.x = fminf(fmaxf(q.x, lo), hi);
          q.y = fminf(fmaxf(q.y, lo), hi);
        }
        int32_t t0, t1;
        magic_rint_bits2(q, t0, t1);
        code[u] = c0 + 4 * k + u < p.c ? t0 + zc : p.out_zero;
        code[u + 1] = c0 + 4 * k + u + 1 < p.c ? t1 + zc : p.out_zero;
      }
      wv[k] = pack_sat_u8x4(code);
    }
    *reinterpret_cast<uint4*>(dst) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
  }
}

// The FP16 depthwise convolution of one kernel row (1 x KW): a CTA 2 x 32 output pixels of one
// row and all channels.  A thread takes one channel pair (half2) over 32 consecutive output
// pixels: its 2 x KW weights in registers, the pair's inputs converted to float once into a
// window of KW registers that slides a pixel at a time; a warp's lanes are 32 consecutive
// pairs, so a pixel's loads and stores are 128 contiguous bytes.  Each output is the generic
// kernel's operations in the same order (an FP32 sum of fmaf over the taps in tap order from 0,
// + bias, ReLU, rounded to FP16): the same bits.
constexpr int kDwF16Run = 32;  // output pixels a thread

template <int KW>
__global__ void __launch_bounds__(256) dw_row_f16_kernel(const __grid_constant__ DwParams p) {
  const int pairs = p.cp >> 1, cpw = p.cp >> 1;  // channel pairs (also the input's half2 a column)
  const int tiles_per_row = (p.ow + 2 * kDwF16Run - 1) / (2 * kDwF16Run);
  const int oy = blockIdx.x / tiles_per_row, ox0 = (blockIdx.x - oy * tiles_per_row) * 2 * kDwF16Run;
  const int sh = p.in_shift;
  const __half2* src = reinterpret_cast<const __half2*>(p.in + static_cast<long long>(oy - p.pt + p.in_ph) * p.in_pitch);
  __half2* dst_row = reinterpret_cast<__half2*>(p.out + static_cast<long long>(oy + p.out_ph) * p.out_pitch);
  for (int it = threadIdx.x; it < 2 * pairs; it += blockDim.x) {
    const int seg = it / pairs, pr = it - seg * pairs;
    const int x0 = ox0 + seg * kDwF16Run;
    if (x0 >= p.ow) continue;
    const int c0 = 2 * pr;
    float w0[KW], w1[KW];
#pragma unroll
    for (int t = 0; t < KW; ++t) {
      w0[t] = __ldg(p.wf + t * p.cp + c0);
      w1[t] = __ldg(p.wf + t * p.cp + c0 + 1);
    }
    const float b0 = __ldg(p.bias + c0), b1 = __ldg(p.bias + c0 + 1);
    const bool in0 = c0 < p.c, in1 = c0 + 1 < p.c;
    auto input = [&](int ox, int t) { return __half22float2(src[static_cast<long long>((ox - p.pl + t) >> sh) * cpw + pr]); };
    float2 win[KW];
#pragma unroll
    for (int t = 0; t < KW; ++t) win[t] = input(x0, t);
#pragma unroll
    for (int j = 0; j < kDwF16Run; ++j) {
      const int ox = x0 + j;
      float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
      for (int t = 0; t < KW; ++t) {
        s0 = __fmaf_rn(win[t].x, w0[t], s0);
        s1 = __fmaf_rn(win[t].y, w1[t], s1);
      }
      float v0 = __fadd_rn(s0, b0), v1 = __fadd_rn(s1, b1);
      if (p.relu) {
        v0 = v0 > 0.0f ? v0 : 0.0f;
        v1 = v1 > 0.0f ? v1 : 0.0f;
      }
      const bool valid = p.mask8[(static_cast<long long>(ox) << p.out_shift) >> 3] != 0;
      dst_row[static_cast<long long>(ox) * cpw + pr] =
          __floats2half2_rn(valid && in0 ? v0 : 0.0f, valid && in1 ? v1 : 0.0f);
      if (j + 1 == kDwF16Run || ox + 1 >= p.ow) break;
#pragma unroll
      for (int t = 0; t + 1 < KW; ++t) win[t] = win[t + 1];
      win[KW - 1] = input(ox + 1, KW - 1);
    }
  }
}

// ---------------------------------------------------------------- the head fused with CTC's argmax
//
// A tile is 128 frames (columns of the head's input, one row); the 1x1 head runs over the
// classes a chunk of up to 128 at a time (tcgen05.mma; A loaded once a tile, the chunks'
// weights streamed by bulk copies), each chunk's accumulator in one of four TMEM buffers.
// Sixteen epilogue warps, four for each TMEM lane quarter: the even chunks go to warps 2-5 and
// 10-13, the odd chunks to 6-9 and 14-17 (each half of the chunks with two buffers of its own),
// warps 2-9 a chunk's first part of its classes, 10-17 the second.
// Per frame: the best class, ties to the lower id, and for a non-blank best its softmax
// probability.
// INT8: each class's logit requantized to uint8 exactly as the reference stores the head's
// output (the dense epilogue), the codes kept in shared memory; the probability as
// carbon/src/cpu/kernels.cpp:799-828 computes it: 1 / (the sum in class order of
// exp_neg(table[q_c] - table[q_best])), table[q] = (q - zero) * scale
// (carbon/src/net/net.cpp:1101-1128).  A term depends only on (q_c, q_best), so the 65,536
// possible terms are computed once per model (ctc_terms_kernel, the same float operations) and
// the sums only add them, in class order.  A sum is a chain of `classes` dependent adds, so it
// is not done here, where a tile's few non-blank frames would hold up its 16 epilogue warps:
// each non-blank frame's codes go out to the run's list (nb_codes), and ctc_sums_kernel adds
// them up over the whole GPU.
// FP16: the FP32 logits (sum + bias); each (half, part) keeps an online maximum and sum of 2^x
// terms, the four merged per frame.
// Only each frame's id and probability leave the kernel; the logits are never written.
struct HeadParams {
  CUtensorMap tmap;     // the head's input: (K byte, frame column, row)
  const uint8_t* wimg;  // [chunk][kb][nchunk rows][128 bytes], swizzled
  int nkb, last_steps, classes, nchunk, chunks;  // last_steps: 32-byte K steps in the last K block
  int ow, num_tiles;
  uint32_t a_bytes, b_bytes;  // A: nkb x 16 KB; B: one chunk (nkb blocks)
  const int32_t* off;   // INT8 [chunks * nchunk]: kMagicBits - in_zero * colsum (fast), else in_zero * colsum
  const float* scale;   // INT8: in_scale * weight scale
  const float* bias;
  int out_zero;
  float out_inv_scale;
  int sat;             // INT8: |v * inv_scale| < 2^21 for every frame (the host's bound), so a code may be
                       // rounded first and clamped by the saturating byte pack
  const float* table;  // INT8 [256]: the u8 logits' values
  uint8_t* nb_codes;   // INT8: the run's non-blank frames' class codes, row k at k * nb_row_bytes
  int nb_row_bytes;    // classes rounded up to 16
  int32_t* nb_frame;   // INT8 [listed]: the frame column of list entry k
  int32_t* nb_best;    // INT8 [listed]: its best code
  int nb_region;       // INT8: list entries a CTA owns (CTA b's from b * nb_region on)
  int* nb_count;       // INT8 [grid][2]: each CTA's frames listed and 255 - its smallest best code listed
  const uint8_t* mask8;
  int out_shift;
  int32_t* frame_id;   // [ow]
  float* frame_prob;   // [ow]
  float* logits;       // optional (tests): [ow][classes] each frame's logits as the reference stores them
  int* err;
};

constexpr int kHeadThreads = 576;  // warp 0 TMA, warp 1 MMA and TMEM, warps 2..17 the epilogue
constexpr int kHeadChunk = 128;    // classes a chunk (the MMA's N): four buffers in 512 TMEM columns
constexpr uint32_t kTmemColsHead = 512;

// The INT8 codes' row stride: 16-byte groups, an odd number of them, so that the 32 rows of a
// warp storing the same 16 classes spread over the shared-memory banks.
__host__ __device__ constexpr int head_code_stride(int classes) {
  return ((classes + 15) / 16 | 1) * 16;
}

// Bytes of the head's shared memory after A, B and the codes: barriers, per-class constants (INT8
// offset, scale and bias; FP16 the bias alone), the per-frame merge slots and the list of
// non-blank frames.
__host__ __device__ constexpr int head_tail_bytes(int ncls, bool int8) {
  return 128 + (int8 ? 12 : 4) * ncls + (3 * 512 + 3 * 128 + 4) * 4;
}

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

// terms[b][q] = exp_neg(table[q] - table[b]): a CTC sum's term for class code q when the best
// code is b.  256 blocks of 256 threads.
__global__ void ctc_terms_kernel(const float* table, float* terms) {
  const int b = blockIdx.x, q = threadIdx.x;
  terms[b * 256 + q] = exp_neg_d(__fsub_rn(table[q], table[b]));
}

// The lowest byte of w equal to the byte in every byte of m4, as a bit mask whose lowest set bit
// is that byte's top bit (bytes above it may be flagged too), or 0 if there is none.
__device__ __forceinline__ uint32_t first_byte_eq(uint32_t w, uint32_t m4) {
  const uint32_t v = w ^ m4;
  return (v - 0x01010101u) & ~v & 0x80808080u;
}

template <bool kInt8, bool kFast, bool kSat>
__global__ void __launch_bounds__(kHeadThreads, 1) head_ctc_kernel(const __grid_constant__ HeadParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int cstride = head_code_stride(p.classes);
  uint8_t* sa = smem;                // A: nkb blocks of [128][128]
  uint8_t* sb = sa + p.a_bytes;      // B: 2 chunk buffers
  uint8_t* codes = sb + 2 * p.b_bytes;  // INT8: [128][cstride]
  uint64_t* bars = reinterpret_cast<uint64_t*>(codes + (kInt8 ? 128 * cstride : 0));
  uint64_t* a_full = bars;
  uint64_t* a_empty = bars + 1;
  uint64_t* b_full = bars + 2;    // [2]
  uint64_t* b_empty = bars + 4;   // [2]
  uint64_t* t_full = bars + 6;    // [4] TMEM buffers: 0, 1 the even chunks', 2, 3 the odd chunks'
  uint64_t* t_empty = bars + 10;  // [4]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);
  const int ncls = p.chunks * p.nchunk, nconst = kInt8 ? ncls : 0;
  int32_t* s_off = reinterpret_cast<int32_t*>(bars + 16);  // INT8 [ncls] per-class constants
  float* s_scale = reinterpret_cast<float*>(s_off + nconst);
  float* s_bias = s_scale + nconst;                         // [ncls]
  int32_t* s_hmax = reinterpret_cast<int32_t*>(s_bias + ncls);  // [4][128] each (half, part)'s highest code (FP16: logit)
  int32_t* s_hbest = s_hmax + 512;                              // FP16 [4][128] each (half, part)'s best class
  float* s_hsum = reinterpret_cast<float*>(s_hbest + 512);     // FP16 [4][128] each (half, part)'s sum
  int32_t* nb_row = reinterpret_cast<int32_t*>(s_hsum + 512);  // INT8: the tile's non-blank frames' rows
  int32_t* nb_q = nb_row + 128;                                 // and best codes
  int32_t* s_best = nb_q + 128;                                 // each row's best class
  volatile int32_t* s_count = s_best + 128;  // [0] frames listed, [1] abort, [2] their place in the run's list, [3] 255 - least best
  __shared__ float tab[256];

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  for (int j = threadIdx.x; j < ncls; j += blockDim.x) {
    if constexpr (kInt8) {
      s_off[j] = p.off[j];
      s_scale[j] = p.scale[j];
    }
    s_bias[j] = p.bias[j];
  }
  if (threadIdx.x < 4) s_count[threadIdx.x] = 0;
  for (int i = threadIdx.x; i < 256; i += blockDim.x) tab[i] = kInt8 ? p.table[i] : 0.0f;
  if (threadIdx.x == 0) {
    mbar_init(a_full, 1);
    mbar_init(a_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&b_empty[i], 1);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&t_full[i], 1);
      mbar_init(&t_empty[i], 8);
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
      uint32_t a_phase = 0, b_phases = 0;  // bit i: B buffer i's phase
      int bi = 0;
      for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
        if (!mbar_wait(a_empty, a_phase ^ 1, p.err, kErrTimeoutEmpty)) break;
        a_phase ^= 1;
        mbar_expect_tx(a_full, p.a_bytes);
        for (int kb = 0; kb < p.nkb; ++kb) tma_load_3d(sa + kb * 16384, &p.tmap, kb * 128, t * 128, 0, a_full);
        bool ok = true;
        for (int c = 0; c < p.chunks; ++c) {
          if (!mbar_wait(&b_empty[bi], ((b_phases >> bi) & 1) ^ 1, p.err, kErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          b_phases ^= 1u << bi;
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
      uint32_t a_phase = 0, b_phases = 0, t_phases = 0, tsel = 0;  // bit i: buffer i's phase; bit h: half h's buffer
      int bi = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
        if (!mbar_wait(a_full, a_phase, p.err, kErrTimeoutFull)) break;
        a_phase ^= 1;
        for (int c = 0; c < p.chunks; ++c) {
          const int half = c & 1, tb = 2 * half + ((tsel >> half) & 1);
          if (!mbar_wait(&t_empty[tb], ((t_phases >> tb) & 1) ^ 1, p.err, kErrTimeoutTmemEmpty) ||
              !mbar_wait(&b_full[bi], (b_phases >> bi) & 1, p.err, kErrTimeoutFull)) {
            ok = false;
            break;
          }
          t_phases ^= 1u << tb;
          b_phases ^= 1u << bi;
          tc_fence_after();
          const uint32_t d = tmem_base + static_cast<uint32_t>(tb * kHeadChunk);
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
          umma_commit(&t_full[tb]);
          bi ^= 1;
          tsel ^= 1u << half;
        }
        umma_commit(a_empty);
      }
    }
  } else {
    const int quarter = warp & 3, half = ((warp - 2) >> 2) & 1, part = (warp - 2) >> 3;
    const int slot = 2 * half + part;  // this warp's (half, part) in the per-row partials
    const int row = quarter * 32 + lane;
    const int e = threadIdx.x - 64;  // 0..511: this thread's place among the epilogue's
    uint32_t t_phases = 0;  // bit i: this half's buffer i's phase
    int tsel = 0;
    const float lo = static_cast<float>(-p.out_zero), hi = static_cast<float>(255 - p.out_zero);
    const int32_t zc = p.out_zero - kMagicBits;
    constexpr float kLog2e = 1.44269504088896341f;
    uint8_t* my = codes + row * cstride;
    bool ok = true;
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
      const int ox = t * 128 + row;
      int32_t mx = -1;                                  // INT8: this part's highest code
      int fi = 0;                                       // INT8: the first class holding it
      float fm = -INFINITY, fsum = 0.0f;                // FP16: this half's highest logit and sum
      int fbest = 0;
      for (int c = half; c < p.chunks && ok; c += 2) {
        const int tb = 2 * half + tsel;
        if (!mbar_wait(&t_full[tb], (t_phases >> tsel) & 1, p.err, kErrTimeoutTmemFull)) {
          ok = false;
          break;
        }
        t_phases ^= 1u << tsel;
        tsel ^= 1;
        tc_fence_after();
        const int cbase = c * p.nchunk;
        // 16 classes from r[0..16), the first j0
        auto take16 = [&](const uint32_t* r, int j0) {
          if constexpr (kInt8) {
            int32_t code[16];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const int4 o = *reinterpret_cast<const int4*>(s_off + j0 + 4 * k);
              const float4 sc = *reinterpret_cast<const float4*>(s_scale + j0 + 4 * k);
              const float4 bb = *reinterpret_cast<const float4*>(s_bias + j0 + 4 * k);
              const int32_t oo[4] = {o.x, o.y, o.z, o.w};
              const float ss[4] = {sc.x, sc.y, sc.z, sc.w}, bv[4] = {bb.x, bb.y, bb.z, bb.w};
#pragma unroll
              for (int u = 0; u < 4; u += 2) {
                // carbon/src/net/net.cpp:703-720: (acc - zero * colsum) * scale + bias, requantized;
                // two classes at a time on the packed FP32 pipe (the same roundings); with kSat the
                // clamp is the saturating pack below (rounding and clamping to integer bounds commute
                // where |q| < 2^21)
                const int32_t a0 = static_cast<int32_t>(r[4 * k + u]), a1 = static_cast<int32_t>(r[4 * k + u + 1]);
                const float2 f = kFast ? magic_to_float2(a0 + oo[u], a1 + oo[u + 1]) : exact_i2f2(a0 - oo[u], a1 - oo[u + 1]);
                float2 q = fmul_pair_rn(fadd2_rn(fmul_pair_rn(f, make_float2(ss[u], ss[u + 1])), make_float2(bv[u], bv[u + 1])),
                                    make_float2(p.out_inv_scale, p.out_inv_scale));
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
            uint4 packed;
            uint32_t* pw = reinterpret_cast<uint32_t*>(&packed);
#pragma unroll
            for (int k = 0; k < 4; ++k) pw[k] = pack_sat_u8x4(code + 4 * k);  // in [0, 255] already without kSat
            *reinterpret_cast<uint4*>(my + j0) = packed;
            if (j0 + 16 > p.classes) {  // classes past the last: out of the maximum (code 0)
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const int keep = p.classes - j0 - 4 * k;  // bytes of word k that are real classes
                pw[k] &= keep >= 4 ? 0xffffffffu : keep <= 0 ? 0u : (1u << (8 * keep)) - 1u;
              }
            }
            // the highest code: byte-wise maxima of the four words, then of the last word's bytes
            uint32_t m4 = __vmaxu4(__vmaxu4(pw[0], pw[1]), __vmaxu4(pw[2], pw[3]));
            m4 = __vmaxu4(m4, m4 >> 16);
            const int32_t m16 = static_cast<int32_t>(__vmaxu4(m4, m4 >> 8) & 0xffu);
            if (m16 > mx) {  // a new highest code: the first of this group's classes holding it (the
                             // classes come in increasing order, so the earlier holder is kept on a tie;
                             // bytes past `classes` are 0 here and never come first)
              mx = m16;
              const uint32_t m4b = static_cast<uint32_t>(m16) * 0x01010101u;
              const uint32_t f0 = first_byte_eq(pw[0], m4b), f1 = first_byte_eq(pw[1], m4b);
              const uint32_t f2 = first_byte_eq(pw[2], m4b), f3 = first_byte_eq(pw[3], m4b);
              fi = j0 + (f0   ? (__ffs(f0) - 1) >> 3
                         : f1 ? 4 + ((__ffs(f1) - 1) >> 3)
                         : f2 ? 8 + ((__ffs(f2) - 1) >> 3)
                              : 12 + ((__ffs(f3) - 1) >> 3));
            }
          } else {
            float v[16];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const float4 bb = *reinterpret_cast<const float4*>(s_bias + j0 + 4 * k);
              v[4 * k] = __fadd_rn(__uint_as_float(r[4 * k]), bb.x);
              v[4 * k + 1] = __fadd_rn(__uint_as_float(r[4 * k + 1]), bb.y);
              v[4 * k + 2] = __fadd_rn(__uint_as_float(r[4 * k + 2]), bb.z);
              v[4 * k + 3] = __fadd_rn(__uint_as_float(r[4 * k + 3]), bb.w);
            }
            if (j0 + 16 > p.classes) {
#pragma unroll
              for (int i = 0; i < 16; ++i)
                if (j0 + i >= p.classes) v[i] = -INFINITY;
            }
            if (p.logits && ox < p.ow) {
#pragma unroll
              for (int i = 0; i < 16; ++i)
                if (j0 + i < p.classes) p.logits[static_cast<long long>(ox) * p.classes + j0 + i] = v[i];
            }
            float m8[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) m8[i] = fmaxf(v[i], v[i + 8]);
#pragma unroll
            for (int i = 0; i < 4; ++i) m8[i] = fmaxf(m8[i], m8[i + 4]);
            const float mb = fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3]));
            if (mb > fm) {  // a new best: the first class holding it; the sum so far rescaled
              int idx = 15;
#pragma unroll
              for (int i = 14; i >= 0; --i) idx = v[i] == mb ? i : idx;
              fsum = fm == -INFINITY ? 0.0f : fsum * ex2_approx((fm - mb) * kLog2e);
              fm = mb;
              fbest = j0 + idx;
            }
            const float fl = fm * kLog2e;
#pragma unroll
            for (int i = 0; i < 16; ++i) fsum += ex2_approx(fmaf(v[i], kLog2e, -fl));
          }
        };
        // this part's 16-class groups of the chunk, [g0, g1) (the first part an even count), read
        // 32 columns at a time (the other warps hide the loads' latency); the buffer goes back to
        // the MMA as soon as the part's last load has completed (a warp without groups has still
        // waited for the buffer, so that its arrival counts for this use)
        const int groups = min(p.nchunk, (p.classes - cbase + 15) & ~15) >> 4;
        const int gsplit = ((groups + 3) >> 2) << 1;
        const int g0 = part ? min(gsplit, groups) : 0, g1 = part ? groups : min(gsplit, groups);
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                               static_cast<uint32_t>(tb * kHeadChunk);
        auto release = [&]() {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&t_empty[tb]);
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
          take16(ra, cbase + g * 16);
          if (w == 2) take16(ra + 16, cbase + g * 16 + 16);
        }
      }
      // the four (half, part) partials of each frame meet
      if (!ok) s_count[1] = 1;
      if constexpr (kInt8) {
        s_hmax[slot * 128 + row] = mx;
        s_hbest[slot * 128 + row] = fi;
      } else {
        s_hmax[slot * 128 + row] = __float_as_int(fm);
        s_hbest[slot * 128 + row] = fbest;
        s_hsum[slot * 128 + row] = fsum;
      }
      named_bar(1, 512);
      if (s_count[1]) break;
      const bool valid = ox < p.ow && p.mask8[(static_cast<long long>(ox) << p.out_shift) >> 3] != 0;
      if (slot == 0) {
        if constexpr (kInt8) {
          // the highest code and the first class holding it (ties: the lower class, as
          // carbon/src/cpu/kernels.cpp:799-828 takes it): the lowest first class among the parts
          // whose highest code it is
          const int32_t m = max(max(s_hmax[row], s_hmax[128 + row]), max(s_hmax[256 + row], s_hmax[384 + row]));
          int best = 0x7fffffff;
#pragma unroll
          for (int i = 0; i < 4; ++i)
            if (s_hmax[i * 128 + row] == m) best = min(best, s_hbest[i * 128 + row]);
          s_best[row] = best;
          if (valid && best != 0) {
            const int k = atomicAdd(const_cast<int32_t*>(&s_count[0]), 1);
            nb_row[k] = row;
            nb_q[k] = m;
            atomicMax(const_cast<int32_t*>(&s_count[3]), 255 - m);
          } else if (valid) {
            p.frame_id[ox] = 0;
            p.frame_prob[ox] = 0.0f;
          }
        } else {
          // the highest logit (ties: the lower class) and the partial sums rescaled to it
          int bi = 0;
#pragma unroll
          for (int i = 1; i < 4; ++i) {
            const float mi = __int_as_float(s_hmax[i * 128 + row]), mb = __int_as_float(s_hmax[bi * 128 + row]);
            if (mi > mb || (mi == mb && s_hbest[i * 128 + row] < s_hbest[bi * 128 + row])) bi = i;
          }
          const float top = __int_as_float(s_hmax[bi * 128 + row]);
          float sum = 0.0f;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float mi = __int_as_float(s_hmax[i * 128 + row]);
            if (i == bi) sum += s_hsum[i * 128 + row];
            else if (mi != -INFINITY) sum += s_hsum[i * 128 + row] * ex2_approx((mi - top) * kLog2e);
          }
          const int best = s_hbest[bi * 128 + row];
          if (valid) {
            p.frame_id[ox] = best;
            p.frame_prob[ox] = best != 0 ? __fdiv_rn(1.0f, sum) : 0.0f;
          }
        }
      } else if (kInt8 && slot == 2 && p.logits && ox < p.ow) {  // test hook: the dequantized logits
        for (int j = 0; j < p.classes; ++j) p.logits[static_cast<long long>(ox) * p.classes + j] = tab[my[j]];
      }
      named_bar(1, 512);
      if constexpr (kInt8) {
        // the listed (non-blank) frames to this CTA's part of the run's list: their ids now,
        // their codes for the class-order sums (ctc_sums_kernel)
        const int listed = s_count[0], base = blockIdx.x * p.nb_region + s_count[2];
        const int w16 = p.nb_row_bytes >> 4;
        for (int i = e; i < listed * w16; i += 512) {
          const int k = i / w16, j = i - k * w16;
          *reinterpret_cast<uint4*>(p.nb_codes + static_cast<long long>(base + k) * p.nb_row_bytes + 16 * j) =
              *reinterpret_cast<const uint4*>(codes + nb_row[k] * cstride + 16 * j);
        }
        for (int k = e; k < listed; k += 512) {
          const int fx = t * 128 + nb_row[k];
          p.nb_frame[base + k] = fx;
          p.nb_best[base + k] = nb_q[k];
          p.frame_id[fx] = s_best[nb_row[k]];
        }
        named_bar(1, 512);
        if (e == 0) {  // read by every thread before the barrier; the next list follows the next one
          s_count[2] = s_count[2] + listed;
          s_count[0] = 0;
        }
      }
    }
    if (kInt8 && e == 0) {  // this CTA's list for the sums
      p.nb_count[2 * blockIdx.x] = s_count[2];
      p.nb_count[2 * blockIdx.x + 1] = s_count[3];
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kTmemColsHead);
}

// ---------------------------------------------------------------- class-order sums
//
// The probability of each listed (non-blank) frame: 1 / (the sum over classes, in class order, of
// terms[best][q_c]) (carbon/src/cpu/kernels.cpp:799-828), a thread a frame.  The terms rows of
// the best codes a run lists (codes from the least listed one up, at most kSumRows rows) are
// staged in shared memory, so the chain of dependent adds reads its terms there; a frame whose
// best code is below them reads its row from global memory.  The staged rows are kSumPitch floats
// apart, one more than a row: the warp's frames look up the same class at once, and their codes
// for it cluster, so with a pitch of 256 the lookups of different rows would fall in one bank.
constexpr int kSumRows = 192;
constexpr int kSumPitch = 257;
constexpr int kSumThreads = 512;

template <bool kShared>
__device__ __forceinline__ float class_sum(const uint8_t* row, int classes, const float* trow) {
  float sum = 0.0f;
  const uint4* r4 = reinterpret_cast<const uint4*>(row);
  const int nfull = classes >> 4;
  // the next four 16-code chunks in flight (a ring of registers), so the chain of adds does not
  // wait on each chunk's load; the chunks are added in class order
  constexpr int kAhead = 4;
  uint4 ring[kAhead];
#pragma unroll
  for (int a = 0; a < kAhead; ++a) ring[a] = a < nfull ? __ldg(r4 + a) : make_uint4(0, 0, 0, 0);
  for (int c = 0; c < nfull; c += kAhead) {
#pragma unroll
    for (int a = 0; a < kAhead; ++a) {
      if (c + a >= nfull) break;
      const uint4 cur = ring[a];
      if (c + a + kAhead < nfull) ring[a] = __ldg(r4 + c + a + kAhead);
      const uint32_t ww[4] = {cur.x, cur.y, cur.z, cur.w};
      float t[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const uint32_t q = (ww[i >> 2] >> (8 * (i & 3))) & 0xffu;
        t[i] = kShared ? trow[q] : __ldg(trow + q);
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) sum = __fadd_rn(sum, t[i]);
    }
  }
  for (int j = nfull << 4; j < classes; ++j) {
    const uint32_t q = row[j];
    sum = __fadd_rn(sum, kShared ? trow[q] : __ldg(trow + q));
  }
  return sum;
}

// CTA b takes the list part the head's CTA b wrote (the same grid).
__global__ void __launch_bounds__(kSumThreads) ctc_sums_kernel(const uint8_t* nb_codes, int row_bytes,
                                                               const int32_t* nb_frame, const int32_t* nb_best,
                                                               const int* nb_count, int nb_region, const float* terms,
                                                               int classes, float* frame_prob) {
  extern __shared__ __align__(16) float srows[];  // [rows][kSumPitch]: terms rows lo .. 255
  const int count = nb_count[2 * blockIdx.x];
  if (count == 0) return;
  const int lo = max(255 - nb_count[2 * blockIdx.x + 1], 256 - kSumRows);
  const long long first = static_cast<long long>(blockIdx.x) * nb_region;
  const float4* src = reinterpret_cast<const float4*>(terms + static_cast<size_t>(lo) * 256);
  for (int i = threadIdx.x; i < (256 - lo) * 64; i += blockDim.x) {
    const float4 v = __ldg(src + i);
    float* d = srows + (i >> 6) * kSumPitch + (i & 63) * 4;
    d[0] = v.x;
    d[1] = v.y;
    d[2] = v.z;
    d[3] = v.w;
  }
  __syncthreads();
  for (long long k = first + threadIdx.x; k < first + count; k += blockDim.x) {
    const int b = nb_best[k];
    const uint8_t* row = nb_codes + k * row_bytes;
    const float sum = b >= lo ? class_sum<true>(row, classes, srows + (b - lo) * kSumPitch)
                              : class_sum<false>(row, classes, terms + static_cast<size_t>(b) * 256);
    frame_prob[nb_frame[k]] = __fdiv_rn(1.0f, sum);
  }
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
  // the frames' ids and probabilities eight at a time, loaded before any of the eight is written
  // out (the outputs are other arrays, but the compiler cannot know that, so a load after a store
  // would wait for it); the current character's highest probability kept in a register
  const int32_t* __restrict__ fid = p.frame_id + f0;
  const float* __restrict__ fpr = p.frame_prob + f0;
  int k = 0, prev = 0;
  float best = 0.0f;
  for (int t0 = 0; t0 < len; t0 += 8) {
    int32_t id8[8];
    float q8[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      id8[u] = t0 + u < len ? __ldg(fid + t0 + u) : 0;
      q8[u] = t0 + u < len ? __ldg(fpr + t0 + u) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      if (t0 + u >= len) break;
      const int id = id8[u];
      const float q = q8[u];
      if (id != 0 && id != prev) {
        if (k > 0) p.probs[f0 + k - 1] = best;
        p.ids[f0 + k] = id;
        p.frames[f0 + k] = t0 + u;
        best = q;
        ++k;
      } else if (id != 0) {
        best = best > q ? best : q;
      }
      prev = id;
    }
  }
  if (k > 0) p.probs[f0 + k - 1] = best;
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

