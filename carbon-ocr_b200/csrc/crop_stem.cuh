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

constexpr int kCropThreads = 256;
constexpr int kMaxTaps = 32;        // taps a sample may have: downscales up to 15x (the host checks)
constexpr int kStripBytes = 48 << 10;  // the horizontal pass's intermediate: source rows x strip columns
constexpr int kMaxStripCols = 256;  // output columns a horizontal strip at most
constexpr int kMaxSrcRows = 1024;   // source rows a crop's vertical windows may span (the host checks)
constexpr int kStemOut = 32;        // the stem's output channels this kernel supports (padded)

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
  // stem: 3x3 (kh x kw), stride (sh, sw), pads (pt, pl), one input channel
  int kh, kw, sh, sw, pt, pl;
  int cout, cp_out;
  const int8_t* w8;     // [cout][kh*kw]
  const float* wf;      // [cout][kh*kw] (FP16 engine: the weights' float16 values widened)
  const float* scale;   // [cout]
  const float* bias;    // [cout]
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
// returns the first source index, the count in *n, the fixed-point weights in k.
__device__ __forceinline__ int coeffs(double in0, double in1, int out, int xx, int32_t (&k)[kMaxTaps], int* n) {
  const double scale = __ddiv_rn(__dsub_rn(in1, in0), static_cast<double>(out));
  const double fs = scale < 1.0 ? 1.0 : scale;
  const double support = __dmul_rn(1.0, fs), ss = __ddiv_rn(1.0, fs);
  const double center = __dadd_rn(in0, __dmul_rn(__dadd_rn(static_cast<double>(xx), 0.5), scale));
  const int xmin = floor_i(__dadd_rn(__dsub_rn(center, support), 0.5));
  int cnt = floor_i(__dadd_rn(__dadd_rn(center, support), 0.5)) - xmin;
  if (cnt > kMaxTaps) cnt = kMaxTaps;  // never at the supported scales (checked by the host)
  double ww = 0.0;
  for (int x = 0; x < cnt; ++x)
    ww = __dadd_rn(ww, tri(__dmul_rn(__dadd_rn(__dsub_rn(static_cast<double>(x + xmin), center), 0.5), ss)));
#pragma unroll
  for (int x = 0; x < kMaxTaps; ++x) {
    if (x < cnt) {
      double w = tri(__dmul_rn(__dadd_rn(__dsub_rn(static_cast<double>(x + xmin), center), 0.5), ss));
      if (ww != 0.0) w = __ddiv_rn(w, ww);
      const double f = static_cast<double>(1 << 22);
      k[x] = static_cast<int32_t>(w < 0 ? __dadd_rn(-0.5, __dmul_rn(w, f)) : __dadd_rn(0.5, __dmul_rn(w, f)));
    } else {
      k[x] = 0;
    }
  }
  *n = cnt;
  return xmin;
}

__device__ __forceinline__ uint8_t clip8d(int32_t v) {
  v >>= 22;
  return static_cast<uint8_t>(v < 0 ? 0 : v > 255 ? 255 : v);
}

// Shared memory: crop [height][bw] | strip intermediate (kStripBytes: source rows x strip columns) |
// vertical coefficients | histogram and counters.
template <bool kInt8>
__global__ void __launch_bounds__(kCropThreads) crop_stem_kernel(const __grid_constant__ CropParams p) {
  extern __shared__ __align__(16) uint8_t sm[];
  const int line = blockIdx.x;
  const LineDesc L = p.lines[line];
  const PageDesc P = p.pages[L.page];
  const int H = p.height, bw = L.bw, cw = L.width;
  uint8_t* crop = sm;                                    // [H][bw]
  uint8_t* tmp = crop + ((H * bw + 15) & ~15);           // [rows][strip columns], kStripBytes
  int32_t* vk = reinterpret_cast<int32_t*>(tmp + kStripBytes);  // [H][kMaxTaps]
  int32_t* vfirst = vk + H * kMaxTaps;                   // [H]
  int32_t* vcount = vfirst + H;                          // [H]
  int32_t* hist = vcount + H;                            // [256]
  int32_t* red = hist + 256;                             // reductions
  const int tid = threadIdx.x;

  if (p.crops_in) {  // a ready crop (already finished and padded to its bucket width)
    const uint8_t* src = p.crops_in + static_cast<long long>(line) * H * p.crops_in_pitch;
    for (int i = tid; i < H * bw; i += blockDim.x) crop[i] = src[(i / bw) * p.crops_in_pitch + i % bw];
    __syncthreads();
  } else {
    // vertical coefficients, one thread a row
    for (int yy = tid; yy < H; yy += blockDim.x) {
      int32_t k[kMaxTaps];
      int n;
      vfirst[yy] = coeffs(L.y0, L.y1, H, yy, k, &n);
      vcount[yy] = n;
      for (int i = 0; i < kMaxTaps; ++i) vk[yy * kMaxTaps + i] = k[i];
    }
    for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0;
    if (tid < 8) red[tid] = 0;
    __syncthreads();
    const int top = vfirst[0];
    const int rows = vfirst[H - 1] + vcount[H - 1] - top;
    if (rows > kMaxSrcRows) {
      if (tid == 0) atomicCAS(p.err, 0, kErrBadShape);
      return;
    }

    // resample, a strip of columns at a time (as wide as the intermediate holds for these rows)
    const int strip = max(16, min(kMaxStripCols, (kStripBytes / max(rows, 1)) & ~15));
    for (int x0 = 0; x0 < cw; x0 += strip) {
      const int sc = min(strip, cw - x0);
      for (int xx = tid; xx < sc; xx += blockDim.x) {
        int32_t k[kMaxTaps];
        int n;
        const int xmin = coeffs(L.x0, L.x1, cw, x0 + xx, k, &n);
        for (int r = 0; r < rows; ++r) {
          const int y = top + r;
          const bool row_in = y >= 0 && y < P.height;
          const uint8_t* src = P.data + static_cast<long long>(y) * P.stride;
          int32_t ss = 1 << 21;
  #pragma unroll
          for (int i = 0; i < kMaxTaps; ++i) {
            if (i < n) {
              const int x = xmin + i;
              const int v = (row_in && x >= 0 && x < P.width) ? src[x] : 255;
              ss += v * k[i];
            }
          }
          tmp[r * strip + xx] = clip8d(ss);
        }
      }
      __syncthreads();
      for (int i = tid; i < H * sc; i += blockDim.x) {
        const int yy = i / sc, xx = i % sc;
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
  // line's segment of the stem tensor; then the gap after it
  const int oh = (H + 2 * p.pt - p.kh) / p.sh + 1, ow = (bw + 2 * p.pl - p.kw) / p.sw + 1;
  const int taps = p.kh * p.kw;
  const long long col0 = static_cast<long long>(L.seg) >> p.out_shift;
  const int eb = kInt8 ? 1 : 2;
  for (int i = tid; i < oh * ow; i += blockDim.x) {
    const int oy = i / ow, ox = i % ow;
    float in[9];
    int32_t qin[9];
    for (int t = 0; t < taps && t < 9; ++t) {
      const int y = oy * p.sh - p.pt + t / p.kw, x = ox * p.sw - p.pl + t % p.kw;
      const bool inside = y >= 0 && y < H && x >= 0 && x < bw;
      const uint8_t px = inside ? crop[y * bw + x] : 0;
      if constexpr (kInt8) {
        qin[t] = (inside ? static_cast<int32_t>(p.in_table[px]) : p.in_zero) - p.in_zero;
      } else {
        // the FP16 engine's input: the ink 1 - p / 255 rounded to float16
        in[t] = inside ? __half2float(__float2half_rn(__fsub_rn(1.0f, __fdiv_rn(static_cast<float>(px), 255.0f)))) : 0.0f;
      }
    }
    uint8_t* dst = p.out + (oy + p.out_ph) * p.out_pitch + (col0 + ox) * p.cp_out * eb;
    for (int c0 = 0; c0 < p.cp_out; c0 += 16) {
      if constexpr (kInt8) {
        alignas(16) uint8_t o[16];
        const float lo = static_cast<float>(-p.out_zero), hi = static_cast<float>(255 - p.out_zero);
        for (int u = 0; u < 16; ++u) {
          const int j = c0 + u;
          if (j >= p.cout) {
            o[u] = static_cast<uint8_t>(p.out_zero);
            continue;
          }
          int32_t s = 0;
          for (int t = 0; t < taps; ++t) s += qin[t] * p.w8[j * taps + t];
          float v = __fmul_rn(static_cast<float>(s), p.scale[j]);
          v = __fadd_rn(v, p.bias[j]);
          if (p.relu) v = v > 0.0f ? v : 0.0f;
          float q = __fmul_rn(v, p.out_inv_scale);
          q = q > lo ? q : lo;
          q = q < hi ? q : hi;
          o[u] = static_cast<uint8_t>(__float2int_rn(q) + p.out_zero);
        }
        *reinterpret_cast<uint4*>(dst + c0) = *reinterpret_cast<const uint4*>(o);
      } else {
        alignas(16) __half o[16];
        for (int u = 0; u < 16; ++u) {
          const int j = c0 + u;
          float v = 0.0f;
          if (j < p.cout) {
            for (int t = 0; t < taps; ++t) v = __fmaf_rn(in[t], p.wf[j * taps + t], v);
            v = __fadd_rn(v, p.bias[j]);
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
