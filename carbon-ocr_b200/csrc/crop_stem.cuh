// The crop rule and the recognizer's first convolution, fused: one CTA a line.
//
// 1. Resample the line's region of its page to 32 x width (carbon/src/lines.cpp:119-160, the
//    scalar reference): the triangle filter's coefficients in IEEE double, each operation
//    rounded on its own (__dmul_rn and friends: no contraction), in 22-bit fixed point
//    (carbon/src/resample_math.h:32-77); a horizontal pass over every source row the vertical
//    one reads into an 8-bit intermediate, then the vertical pass.  Pixels off the page read
//    as paper (255).  Columns are processed in strips so the intermediate fits in shared memory.
// 2. Finish it (carbon/src/lines.cpp:249-329): the ground is the median of the first row, the
//    last row and the last column; flip (255 - v) when more bytes are at least flip_margin
//    lighter than the ground than as much darker (and, with flip_needs_dark, over half the
//    bytes are at most 127); pad to the line's bucket width with the (flipped) ground.
// 3. Quantize (INT8: the input table, ink 1 - p / 255 quantized as the graph's input,
//    carbon/src/net/net.cpp:84-90 and carbon/src/pipeline.cpp:153; FP16: the ink as float16)
//    and run the stem (3x3, stride 2, one input channel) straight from shared memory, writing
//    its output into the line's columns of the group's stem tensor, and the zero point into
//    the gap columns after them.
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

#include "sm100.cuh"

namespace crec {

constexpr int kCropThreads = 512;
constexpr int kMaxTaps = 32;          // taps a sample may have: downscales up to 15x (the host checks)
constexpr int kStripBytes = 32 << 10;  // the horizontal pass's intermediate: source rows x strip columns
constexpr int kCoefBytes = 16 << 10;   // a strip's horizontal coefficients: columns x taps x 4 bytes
constexpr int kMaxStripCols = 512;    // output columns a strip at most
constexpr int kMaxSrcRows = 1024;     // source rows a crop's vertical windows may span (the host checks)
constexpr int kStemMaxOut = 64;       // the stem's output channels at most (padded)

struct PageDesc {
  const uint8_t* data;
  int width, height;
  long long stride;
};

struct LineDesc {
  double x0, y0, x1, y1;  // the crop region (crop_region)
  int page, width, bw, seg;  // crop width, bucket width, first column of its segment (input resolution)
  int next_seg;              // first column of the next line's segment (or the group's total)
  int pad_;
};

struct CropParams {
  const PageDesc* pages;
  const LineDesc* lines;
  int n, height, flip_margin, flip_needs_dark;
  uint8_t* crops_out;  // optional: the finished crops [n][height][max_bw] (tests)
  int crops_pitch;     // bytes per crop row in crops_out
  const uint8_t* crops_in;  // optional: crops given ready, [n][height][crops_in_pitch]: no resampling, no finish
  int crops_in_pitch;
  int max_bw;  // the widest bucket of the run (the crop buffer's size in shared memory)
  // stem: 3x3 (kh x kw), stride (sh, sw), pads (pt, pl), one input channel
  int kh, kw, sh, sw, pt, pl;
  int cout, cp_out;
  const int8_t* w8;     // [cout][kh*kw]
  const float* wf;      // [cout][kh*kw] (FP16 engine: the weights' float16 values widened)
  const float* scale;   // [cout]
  const float* bias;    // [cout]
  const int32_t* colsum;  // [cout] sum of each output channel's int8 weights
  const uint8_t* in_table;  // [256] the INT8 input table
  int in_zero, out_zero, relu;
  float out_inv_scale;
  uint8_t* out;  // stem tensor's first row
  int out_ph;
  long long out_pitch;
  int out_shift;  // log2 of input columns per stem column
  int* err;
};

__device__ __forceinline__ double tri(double x) {
  if (x < 0.0) x = -x;
  return x < 1.0 ? __dsub_rn(1.0, x) : 0.0;
}
__device__ __forceinline__ int floor_i(double v) {
  const int i = static_cast<int>(v);
  return i - (v < static_cast<double>(i) ? 1 : 0);
}

// The coefficients of output sample xx of a filter over [in0, in1) to `out` samples:
// returns the first source index, the count in *n (at most kMaxTaps: the host checks the
// scale), the fixed-point weights in k[0 .. n) (shared memory).
__device__ __forceinline__ int coeffs(double in0, double in1, int out, int xx, int32_t* k, int* n) {
  const double scale = __ddiv_rn(__dsub_rn(in1, in0), static_cast<double>(out));
  const double fs = scale < 1.0 ? 1.0 : scale;
  const double support = __dmul_rn(1.0, fs), ss = __ddiv_rn(1.0, fs);
  const double center = __dadd_rn(in0, __dmul_rn(__dadd_rn(static_cast<double>(xx), 0.5), scale));
  const int xmin = floor_i(__dadd_rn(__dsub_rn(center, support), 0.5));
  int cnt = floor_i(__dadd_rn(__dadd_rn(center, support), 0.5)) - xmin;
  if (cnt > kMaxTaps) cnt = kMaxTaps;
  double ww = 0.0;
  for (int x = 0; x < cnt; ++x)
    ww = __dadd_rn(ww, tri(__dmul_rn(__dadd_rn(__dsub_rn(static_cast<double>(x + xmin), center), 0.5), ss)));
  const double f = static_cast<double>(1 << 22);
  for (int x = 0; x < cnt; ++x) {
    double w = tri(__dmul_rn(__dadd_rn(__dsub_rn(static_cast<double>(x + xmin), center), 0.5), ss));
    if (ww != 0.0) w = __ddiv_rn(w, ww);
    k[x] = static_cast<int32_t>(w < 0 ? __dadd_rn(-0.5, __dmul_rn(w, f)) : __dadd_rn(0.5, __dmul_rn(w, f)));
  }
  *n = cnt;
  return xmin;
}

// Round half to even and saturate to [0, 255] (the output stage for a zero point of 0 after a ReLU).
__device__ __forceinline__ uint32_t cvt_rni_sat_u8(float q) {
  uint32_t r;
  asm("cvt.rni.sat.u8.f32 %0, %1;" : "=r"(r) : "f"(q));
  return r;
}

// Four unsigned bytes of a times four signed bytes of b, summed into c.
__device__ __forceinline__ int32_t dp4a_us(uint32_t a, uint32_t b, int32_t c) {
  int32_t d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ uint8_t clip8d(int32_t v) {
  v >>= 22;
  return static_cast<uint8_t>(v < 0 ? 0 : v > 255 ? 255 : v);
}

// Shared memory: crop [height][bw] | strip intermediate (kStripBytes) | a strip's horizontal
// coefficients (kCoefBytes: first and count a column, then taps) | vertical coefficients |
// the stem's weights and per-channel constants | histogram and counters.
template <bool kInt8>
__global__ void __launch_bounds__(kCropThreads) crop_stem_kernel(const __grid_constant__ CropParams p) {
  extern __shared__ __align__(16) uint8_t sm[];
  const int line = blockIdx.x;
  const LineDesc L = p.lines[line];
  const PageDesc P = p.pages[L.page];
  const int H = p.height, bw = L.bw, cw = L.width;
  uint8_t* crop = sm;                                                   // [H][bw]
  uint8_t* tmp = crop + ((H * p.max_bw + 15) & ~15);                    // [rows][strip]
  int32_t* hk = reinterpret_cast<int32_t*>(tmp + kStripBytes);         // [strip][2 + T]
  int32_t* vk = hk + kCoefBytes / 4;                                   // [H][kMaxTaps]
  int32_t* vfirst = vk + H * kMaxTaps;                                 // [H]
  int32_t* vcount = vfirst + H;                                        // [H]
  int32_t* hist = vcount + H;                                          // [256]
  int32_t* red = hist + 256;                                           // [8] reductions
  float* sw_ = reinterpret_cast<float*>(red + 8);                      // stem weights [cout][taps] (FP16 engine)
  float* sscale = sw_ + kStemMaxOut * 9;                               // [cout]
  float* sbias = sscale + kStemMaxOut;                                 // [cout]
  uint32_t* sw4 = reinterpret_cast<uint32_t*>(sbias + kStemMaxOut);    // INT8: [cout][3] taps packed 4 a word
  int32_t* scol = reinterpret_cast<int32_t*>(sw4 + kStemMaxOut * 3);   // [cout] weight sums
  uint8_t* stab = reinterpret_cast<uint8_t*>(scol + kStemMaxOut);      // [256] input table
  const int tid = threadIdx.x;
  const int taps_stem = p.kh * p.kw;

  if (!kInt8)
    for (int i = tid; i < p.cout * taps_stem; i += blockDim.x) sw_[i] = p.wf[i];
  if (kInt8)
    for (int i = tid; i < p.cout * 3; i += blockDim.x) {  // taps 4k .. 4k+3 of channel i / 3, zeros past the last
      const int j = i / 3, k = i % 3;
      uint32_t w = 0;
      for (int b = 0; b < 4; ++b) {
        const int t = 4 * k + b;
        if (t < taps_stem) w |= static_cast<uint32_t>(static_cast<uint8_t>(p.w8[j * taps_stem + t])) << (8 * b);
      }
      sw4[i] = w;
    }
  for (int i = tid; i < p.cout; i += blockDim.x) {
    sscale[i] = kInt8 ? p.scale[i] : 1.0f;
    sbias[i] = p.bias[i];
    scol[i] = kInt8 ? p.colsum[i] : 0;
  }
  if (kInt8)
    for (int i = tid; i < 256; i += blockDim.x) stab[i] = p.in_table[i];
  for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0;
  if (tid < 8) red[tid] = 0;

  if (p.crops_in) {  // a ready crop (already finished and padded to its bucket width)
    const uint8_t* src = p.crops_in + static_cast<long long>(line) * H * p.crops_in_pitch;
    for (int i = tid; i < H * bw; i += blockDim.x) crop[i] = src[(i / bw) * p.crops_in_pitch + i % bw];
    __syncthreads();
  } else {
    // vertical coefficients, one thread a row
    for (int yy = tid; yy < H; yy += blockDim.x) {
      int n;
      vfirst[yy] = coeffs(L.y0, L.y1, H, yy, vk + yy * kMaxTaps, &n);
      vcount[yy] = n;
    }
    __syncthreads();
    const int top = vfirst[0];
    const int rows = vfirst[H - 1] + vcount[H - 1] - top;
    if (rows > kMaxSrcRows) {
      if (tid == 0) atomicCAS(p.err, 0, kErrBadShape);
      return;
    }
    // this line's tap stride: the filter's most taps (PIL's ksize)
    const double hscale = (L.x1 - L.x0) / cw;
    const int T = min(kMaxTaps, static_cast<int>(ceil(hscale < 1.0 ? 1.0 : hscale)) * 2 + 1);
    const int strip = max(16, min(kMaxStripCols, min(kStripBytes / max(rows, 1), kCoefBytes / (4 * (T + 2)))));
    for (int x0 = 0; x0 < cw; x0 += strip) {
      const int sc = min(strip, cw - x0);
      // the strip's horizontal coefficients, a thread a column
      for (int xx = tid; xx < sc; xx += blockDim.x) {
        int32_t* c = hk + xx * (T + 2);
        int n;
        c[0] = coeffs(L.x0, L.x1, cw, x0 + xx, c + 2, &n);
        c[1] = n;
      }
      __syncthreads();
      // horizontal pass: a thread an (intermediate row, column)
      for (int i = tid; i < rows * sc; i += blockDim.x) {
        const int r = i / sc, xx = i - r * sc;
        const int32_t* c = hk + xx * (T + 2);
        const int xmin = c[0], n = c[1];
        const int y = top + r;
        int32_t ss = 1 << 21;
        if (y >= 0 && y < P.height) {
          const uint8_t* src = P.data + static_cast<long long>(y) * P.stride;
          if (xmin >= 0 && xmin + n <= P.width) {
            for (int t = 0; t < n; ++t) ss += static_cast<int32_t>(__ldg(src + xmin + t)) * c[2 + t];
          } else {
            for (int t = 0; t < n; ++t) {
              const int x = xmin + t;
              ss += ((x >= 0 && x < P.width) ? static_cast<int32_t>(__ldg(src + x)) : 255) * c[2 + t];
            }
          }
        } else {
          for (int t = 0; t < n; ++t) ss += 255 * c[2 + t];
        }
        tmp[r * strip + xx] = clip8d(ss);
      }
      __syncthreads();
      // vertical pass: a thread an output pixel
      for (int i = tid; i < H * sc; i += blockDim.x) {
        const int yy = i / sc, xx = i - yy * sc;
        const int f = vfirst[yy] - top, n = vcount[yy];
        int32_t ss = 1 << 21;
        for (int t = 0; t < n; ++t) ss += tmp[(f + t) * strip + xx] * vk[yy * kMaxTaps + t];
        crop[yy * bw + x0 + xx] = clip8d(ss);
      }
      __syncthreads();
    }
  // finish: the ground's histogram (first row, last row, last column)
    for (int x = tid; x < cw; x += blockDim.x) {
      atomicAdd(&hist[crop[x]], 1);
      atomicAdd(&hist[crop[(H - 1) * bw + x]], 1);
    }
    for (int y = tid; y < H; y += blockDim.x) atomicAdd(&hist[crop[y * bw + cw - 1]], 1);
    __syncthreads();
    const int count = 2 * cw + H;
    auto nth = [&](int n, bool flipped) {
      int seen = 0;
      for (int v = 0; v < 256; ++v) {
        seen += hist[flipped ? 255 - v : v];
        if (seen > n) return v;
      }
      return 255;
    };
    auto ground_of = [&](bool flipped) {
      return count % 2 ? nth(count / 2, flipped) : (nth(count / 2 - 1, flipped) + nth(count / 2, flipped)) / 2;
    };
    if (tid == 0) red[0] = ground_of(false);
    __syncthreads();
    bool flip = false;
    if (p.flip_margin > 0) {
      const int g = red[0], lo = g - p.flip_margin, hi = g + p.flip_margin;
      int below = 0, above = 0, dark = 0;
      for (int i = tid; i < H * cw; i += blockDim.x) {
        const int v = crop[(i / cw) * bw + i % cw];
        below += v <= lo;
        above += v >= hi;
        dark += v <= 127;
      }
      for (int o = 16; o > 0; o >>= 1) {
        below += __shfl_xor_sync(0xffffffffu, below, o);
        above += __shfl_xor_sync(0xffffffffu, above, o);
        dark += __shfl_xor_sync(0xffffffffu, dark, o);
      }
      if ((tid & 31) == 0) {
        atomicAdd(&red[1], below);
        atomicAdd(&red[2], above);
        atomicAdd(&red[3], dark);
      }
      __syncthreads();
      flip = red[2] > red[1];
      if (flip && p.flip_needs_dark) flip = 2 * static_cast<long long>(red[3]) > static_cast<long long>(cw) * H;
    }
    if (tid == 0) red[4] = ground_of(flip);
    __syncthreads();
    const uint8_t ground = static_cast<uint8_t>(red[4]);
    for (int i = tid; i < H * bw; i += blockDim.x) {
      const int y = i / bw, x = i % bw;
      uint8_t v = crop[y * bw + x];
      if (x >= cw) {
        v = ground;
      } else if (flip) {
        v = static_cast<uint8_t>(255 - v);
      }
      crop[y * bw + x] = v;
    }
    __syncthreads();
    if (p.crops_out) {
      uint8_t* dst = p.crops_out + static_cast<long long>(line) * H * p.crops_pitch;
      for (int i = tid; i < H * bw; i += blockDim.x)
      if (i % bw < p.crops_pitch) dst[(i / bw) * p.crops_pitch + i % bw] = crop[i];
    }

  }
  // the stem on the quantized crop (its border the input's zero point: real zero), into the
  // line's segment of the stem tensor; a thread an output pixel and all its channels
  const int oh = (H + 2 * p.pt - p.kh) / p.sh + 1, ow = (bw + 2 * p.pl - p.kw) / p.sw + 1;
  const long long col0 = static_cast<long long>(L.seg) >> p.out_shift;
  const int eb = kInt8 ? 1 : 2;
  const bool fast = p.in_zero == 0 && p.out_zero == 0 && p.relu && p.cout == p.cp_out;
  for (int i = tid; i < oh * ow; i += blockDim.x) {
    const int oy = i / ow, ox = i - oy * ow;
    uint8_t* dst = p.out + (oy + p.out_ph) * p.out_pitch + (col0 + ox) * p.cp_out * eb;
    if constexpr (kInt8) {
      // the taps' quantized inputs packed 4 a word (the border reads the zero point: real zero);
      // sum over taps of (a - zero) * w = dp4a(a, w) - zero * sum(w), exact in int32
      uint32_t a4[3] = {0, 0, 0};
      for (int t = 0; t < taps_stem; ++t) {
        const int y = oy * p.sh - p.pt + t / p.kw, x = ox * p.sw - p.pl + t % p.kw;
        const uint32_t q = (y >= 0 && y < H && x >= 0 && x < bw) ? stab[crop[y * bw + x]] : static_cast<uint32_t>(p.in_zero);
        a4[t >> 2] |= q << (8 * (t & 3));
      }
      uint32_t words[kStemMaxOut / 4];
      const float lo = static_cast<float>(-p.out_zero), hi = static_cast<float>(255 - p.out_zero);
      for (int c0 = 0; c0 < p.cp_out; c0 += 4) {
        uint32_t wv = 0;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int j = c0 + u;
          uint32_t code = static_cast<uint32_t>(p.out_zero);
          if (j < p.cout) {
            const uint32_t* w = sw4 + j * 3;
            int32_t sum = dp4a_us(a4[0], w[0], 0);
            sum = dp4a_us(a4[1], w[1], sum);
            sum = dp4a_us(a4[2], w[2], sum);
            sum -= p.in_zero * scol[j];
            float v = __fadd_rn(__fmul_rn(static_cast<float>(sum), sscale[j]), sbias[j]);
            if (fast) {
              code = cvt_rni_sat_u8(__fmul_rn(v, p.out_inv_scale));
            } else {
              if (p.relu) v = v > 0.0f ? v : 0.0f;
              float q = __fmul_rn(v, p.out_inv_scale);
              q = q > lo ? q : lo;
              q = q < hi ? q : hi;
              code = static_cast<uint32_t>(__float2int_rn(q) + p.out_zero);
            }
          }
          wv |= (code & 0xffu) << (8 * u);
        }
        words[c0 >> 2] = wv;
      }
      for (int c0 = 0; c0 < p.cp_out; c0 += 16)
        *reinterpret_cast<uint4*>(dst + c0) =
            make_uint4(words[c0 >> 2], words[(c0 >> 2) + 1], words[(c0 >> 2) + 2], words[(c0 >> 2) + 3]);
    } else {
      float in[9];
      for (int t = 0; t < 9; ++t) {
        in[t] = 0.0f;
        if (t >= taps_stem) continue;
        const int y = oy * p.sh - p.pt + t / p.kw, x = ox * p.sw - p.pl + t % p.kw;
        if (y < 0 || y >= H || x < 0 || x >= bw) continue;  // the border: real zero
        // the FP16 engine's input: the ink 1 - p / 255 rounded to float16
        in[t] = __half2float(__float2half_rn(__fsub_rn(1.0f, __fdiv_rn(static_cast<float>(crop[y * bw + x]), 255.0f))));
      }
      for (int c0 = 0; c0 < p.cp_out; c0 += 16) {
        alignas(16) __half o[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          const int j = c0 + u;
          float v = 0.0f;
          if (j < p.cout) {
            for (int t = 0; t < taps_stem; ++t) v = __fmaf_rn(in[t], sw_[j * taps_stem + t], v);
            v = __fadd_rn(v, sbias[j]);
            if (p.relu) v = v > 0.0f ? v : 0.0f;
          }
          o[u] = __float2half_rn(v);
        }
        *reinterpret_cast<uint4*>(dst + c0 * 2) = *reinterpret_cast<const uint4*>(o);
        *reinterpret_cast<uint4*>(dst + c0 * 2 + 16) = *reinterpret_cast<const uint4*>(o + 8);
      }
    }
  }
  // the gap after this line's segment (and before the first line's), the zero point
  const long long gap0 = col0 + ow, gap1 = static_cast<long long>(L.next_seg) >> p.out_shift;
  const long long lead = line == 0 ? col0 : 0;
  const long long gapn = (gap1 - gap0) + lead;
  const int vec = p.cp_out * eb / 16;
  const uint32_t zb = kInt8 ? static_cast<uint32_t>(p.out_zero) * 0x01010101u : 0u;
  const uint4 z4 = make_uint4(zb, zb, zb, zb);
  for (long long i = tid; i < gapn * oh * vec; i += blockDim.x) {
    const long long v = i % vec, rest = i / vec;
    const long long c = rest % gapn, oy = rest / gapn;
    const long long col = c < lead ? c : gap0 + (c - lead);
    *reinterpret_cast<uint4*>(p.out + (oy + p.out_ph) * p.out_pitch + col * p.cp_out * eb + v * 16) = z4;
  }
}

}  // namespace crec
