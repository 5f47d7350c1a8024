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
#include <type_traits>

#include "sm100.cuh"

namespace crec {

constexpr int kCropThreads = 512;
constexpr int kMaxTaps = 32;          // taps a sample may have: downscales up to 15x (the host checks)
constexpr int kStripBytes = 32 << 10;  // the horizontal pass's intermediate: source rows x strip columns
constexpr int kCoefBytes = 16 << 10;   // a strip's horizontal coefficients: columns x taps x 4 bytes
constexpr int kMaxStripCols = 256;    // output columns a strip at most (two row groups keep all 512 threads busy)
constexpr int kMaxSrcRows = 1024;     // source rows a crop's vertical windows may span (the host checks)
constexpr int kStemMaxOut = 64;       // the stem's output channels at most (padded)
constexpr int kMaxHWords = 5;         // horizontal windows of up to 20 taps in the dp4a pass (wider: the generic one)

struct PageDesc {
  const uint8_t* data;
  int width, height;
  long long stride;
};

struct LineDesc {
  double x0, y0, x1, y1;  // the crop region (crop_region)
  int page, width, bw, seg;  // crop width, bucket width, first column of its segment (input resolution)
  int next_seg;              // first column of the next line's segment (or the group's total)
  int wide;                  // -1, or the line's slot in the wide crops (resampled by crop_wide_kernel)
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
  int sat;  // INT8: |v * inv_scale| < 2^21 for every output and no ReLU above a zero point (round,
           // then clamp to [0, 255] while packing)
  float out_inv_scale;
  uint8_t* out;  // stem tensor's first row
  int out_ph;
  long long out_pitch;
  int out_shift;  // log2 of input columns per stem column
  int* err;
  int* claim;  // [2] lines claimed past the first wave, CTAs done: both 0 between launches
  const int* order;  // [n] the lines in the order they are claimed (the costliest first)
  const uint8_t* wide;  // the wide lines' resampled crops, [slot][height][wide_pitch]
  int wide_pitch;
};

// The lines beyond the fast resampler's reach (more than kMaxTaps taps a sample, or more than
// kMaxSrcRows source rows): resampled by crop_wide_kernel into raw crops in global memory, which
// crop_stem_kernel then finishes like its own.
struct WideParams {
  const PageDesc* pages;
  const LineDesc* lines;
  const int* index;  // the run's wide lines, in slot order
  int height;
  int vtaps, htaps;  // vertical / horizontal taps a sample at most (PIL's ksize over the lines)
  int hk_cols;       // columns of horizontal coefficients a strip
  int tmp_bytes;     // the intermediate: source rows x strip columns
  uint8_t* out;      // [slot][height][pitch]
  int pitch;
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
// returns the first source index, the count in *n, the fixed-point weights in k[0 .. n) (shared
// memory).  The count is at most PIL's ksize, 2 ceil(support) + 1 (the windows' bound), and the
// callers check that ksize is within max_taps before they call.
__device__ __forceinline__ int coeffs(double in0, double in1, int out, int xx, int32_t* k, int* n, int max_taps = kMaxTaps) {
  const double scale = __ddiv_rn(__dsub_rn(in1, in0), static_cast<double>(out));
  const double fs = scale < 1.0 ? 1.0 : scale;
  const double support = __dmul_rn(1.0, fs), ss = __ddiv_rn(1.0, fs);
  const double center = __dadd_rn(in0, __dmul_rn(__dadd_rn(static_cast<double>(xx), 0.5), scale));
  const int xmin = floor_i(__dadd_rn(__dsub_rn(center, support), 0.5));
  int cnt = floor_i(__dadd_rn(__dadd_rn(center, support), 0.5)) - xmin;
  if (cnt > max_taps) cnt = max_taps;
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

// Four unsigned bytes of a times four unsigned bytes of b, summed into c.
__device__ __forceinline__ uint32_t dp4a_uu(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ uint8_t clip8d(int32_t v) {
  v >>= 22;
  return static_cast<uint8_t>(v < 0 ? 0 : v > 255 ? 255 : v);
}

// Shared memory, in this order: the crop with a border (qb: [height + 4][qpitch], crop pixel
// (y, x) at row y + 2, column x + 4; the border holds the INT8 input's zero point, the stem's
// padding) | the strip intermediate (kStripBytes) | a strip's horizontal coefficients
// (kCoefBytes: first and count a column, then taps) | the stem's weights and per-channel
// constants | vertical coefficients | histogram, counters and tables.
struct CropSmem {
  int qpitch;
  unsigned qb, tmp, hk, wq, swf, soff, sscale, sbias, vk, vkp, vfirst, vcount, hist, red, ftab, stab, total;
};

__host__ __device__ inline CropSmem crop_smem(int height, int max_bw) {
  CropSmem s{};
  s.qpitch = (max_bw + 12 + 15) & ~15;
  unsigned o = 0;
  s.qb = o;
  o += static_cast<unsigned>((height + 4) * s.qpitch);
  s.tmp = o;
  o += kStripBytes;
  s.hk = o;
  o += kCoefBytes;
  s.wq = o;  // INT8 [cout][3] a kernel row's taps, 4 bytes a row
  o += kStemMaxOut * 3 * 4;
  s.swf = o;  // FP16 [cout][taps]
  o += kStemMaxOut * 9 * 4;
  s.soff = o;
  o += kStemMaxOut * 4;
  s.sscale = o;
  o += kStemMaxOut * 4;
  s.sbias = o;
  o += kStemMaxOut * 4;
  s.vk = o;
  o += static_cast<unsigned>(height * kMaxTaps * 4);
  s.vkp = o;  // the vertical weights' byte planes: [height][3][8] words
  o += static_cast<unsigned>(height * 24 * 4);
  s.vfirst = o;
  o += static_cast<unsigned>(height * 4);
  s.vcount = o;
  o += static_cast<unsigned>(height * 4);
  s.hist = o;
  o += 256 * 4;
  s.red = o;
  o += 8 * 4;
  s.ftab = o;
  o += 256 * 4;
  s.stab = o;
  o += 256;
  s.total = o;
  return s;
}

// The value of the n-th (from 0) byte of a 256-bin histogram in increasing order of value (of
// 255 - value when flipped), 255 if there are not that many; warp-wide, every lane returns it.
__device__ __forceinline__ int hist_nth(const int32_t* hist, int n, bool flipped) {
  const int lane = threadIdx.x & 31;
  int c[8], s = 0;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int v = lane * 8 + k;
    c[k] = hist[flipped ? 255 - v : v];
    s += c[k];
  }
  int incl = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  const int excl = incl - s;
  const uint32_t hit = __ballot_sync(0xffffffffu, excl <= n && n < incl);
  if (hit == 0) return 255;
  int v = lane * 8 + 7, run = excl;  // in the lane that holds it: the first k whose running count passes n
  bool found = false;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    run += c[k];
    if (!found && run > n) {
      v = lane * 8 + k;
      found = true;
    }
  }
  return __shfl_sync(0xffffffffu, v, __ffs(hit) - 1);
}

// The byte planes of a window's 22-bit weights (non-negative): k0 / k1 / k2 hold bits 0-7 /
// 8-15 / 16-23 of taps 4j .. 4j+3 in word j, zero past the window's n taps.
template <int NW>
__device__ __forceinline__ void weight_planes(const int32_t* k, int n, uint32_t (&k0)[NW], uint32_t (&k1)[NW], uint32_t (&k2)[NW]) {
#pragma unroll
  for (int j = 0; j < NW; ++j) {
    uint32_t a = 0, b = 0, d = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int t = 4 * j + i;
      const uint32_t w = t < n ? static_cast<uint32_t>(k[t]) : 0u;
      a |= (w & 0xffu) << (8 * i);
      b |= ((w >> 8) & 0xffu) << (8 * i);
      d |= ((w >> 16) & 0xffu) << (8 * i);
    }
    k0[j] = a;
    k1[j] = b;
    k2[j] = d;
  }
}

// 2^21 plus a window's bytes times its weights: the bytes realigned from the words w[0 .. NW] by
// the byte permute `sel`, four taps a dp4a on each weight plane.  The three plane sums recombine
// modulo 2^32 to the integer sum, which is below 255 * 2^22 * (1 + 2^-20) and so exact.
template <int NW>
__device__ __forceinline__ int32_t window_sum(const uint32_t (&w)[NW + 1], uint32_t sel, const uint32_t (&k0)[NW],
                                              const uint32_t (&k1)[NW], const uint32_t (&k2)[NW]) {
  uint32_t s0 = 0, s1 = 0, s2 = 0;
#pragma unroll
  for (int j = 0; j < NW; ++j) {
    const uint32_t x = __byte_perm(w[j], w[j + 1], sel);
    s0 = dp4a_uu(x, k0[j], s0);
    s1 = dp4a_uu(x, k1[j], s1);
    s2 = dp4a_uu(x, k2[j], s2);
  }
  return (1 << 21) + static_cast<int32_t>(s0 + (s1 << 8) + (s2 << 16));
}

// Four window sums as the intermediate's bytes: >> 22, saturated to [0, 255] (clip8d).
__device__ __forceinline__ uint32_t clip8x4(const int32_t* v) {
  const int32_t c[4] = {v[0] >> 22, v[1] >> 22, v[2] >> 22, v[3] >> 22};
  return pack_sat_u8x4(c);
}

// Horizontal pass of one output column over source rows in chunks of 8 (chunk ch: rows
// top + 8 ch .. + 7), every tap window at most 4 * NW taps and its word reads on the page
// (checked by the caller).  The column of the intermediate is contiguous (col[r] = row r), so a
// chunk is stored as two words.  Rows off the page read as paper.  kSameSel: the page's rows
// are 4-byte aligned, so every row's window has the same byte offset within its first word.
template <int NW, bool kSameSel>
__device__ __forceinline__ void hpass(const PageDesc& P, const int32_t* c, int32_t paper, int top, int first, int nchunks,
                                      int step, uint8_t* col) {
  const int xmin = c[0], n = c[1];
  uint32_t k0[NW], k1[NW], k2[NW];
  weight_planes<NW>(c + 2, n, k0, k1, k2);
  constexpr int RU = NW <= 2 ? 8 : NW <= 4 ? 4 : 2;  // rows whose loads are in flight together
  const uintptr_t a0 = reinterpret_cast<uintptr_t>(P.data + xmin);
  const uint32_t sel0 = 0x3210u + static_cast<uint32_t>(a0 & 3) * 0x1111u;
  const uint32_t* base = reinterpret_cast<const uint32_t*>(a0 & ~uintptr_t(3));
  const long long wstride = P.stride >> 2;
  auto row_words = [&](int y, uint32_t (&w)[NW + 1], uint32_t& sel) {
    const uint32_t* wp;
    if (kSameSel) {
      wp = base + static_cast<long long>(y) * wstride;
      sel = sel0;
    } else {
      const uintptr_t a = a0 + static_cast<uintptr_t>(static_cast<long long>(y) * P.stride);
      wp = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
      sel = 0x3210u + static_cast<uint32_t>(a & 3) * 0x1111u;
    }
#pragma unroll
    for (int j = 0; j <= NW; ++j) w[j] = __ldg(wp + j);
  };
  for (int ch = first; ch < nchunks; ch += step) {
    const int y0 = top + ch * 8;
    int32_t v[8];
    if (y0 >= 0 && y0 + 8 <= P.height) {
#pragma unroll
      for (int h = 0; h < 8; h += RU) {
        uint32_t w[RU][NW + 1], sel[RU];
#pragma unroll
        for (int q = 0; q < RU; ++q) row_words(y0 + h + q, w[q], sel[q]);
#pragma unroll
        for (int q = 0; q < RU; ++q) v[h + q] = window_sum<NW>(w[q], sel[q], k0, k1, k2);
      }
    } else {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int y = y0 + q;
        v[q] = (1 << 21) + paper;
        if (y >= 0 && y < P.height) {
          uint32_t w[NW + 1], sel;
          row_words(y, w, sel);
          v[q] = window_sum<NW>(w, sel, k0, k1, k2);
        }
      }
    }
    uint32_t* o = reinterpret_cast<uint32_t*>(col + ch * 8);
    o[0] = clip8x4(v);
    o[1] = clip8x4(v + 4);
  }
}

// Vertical pass of a strip, a thread an output row and every tpr-th column of the strip from c0
// (tpr threads a row): the row's weight planes stay in registers across its columns.  Column xx's
// intermediate is at tmp + xx * rp; row yy's window at vfirst[yy] - top; the output pixel (yy, xx)
// at out0[yy * qpitch + xx]; every window at most 4 * NW taps, its word reads inside the column's slot.
template <int NW>
__device__ __forceinline__ void vpass_rows(const uint8_t* tmp, int rp, const int32_t* vfirst, const uint32_t* vkp,
                                           int top, int yy, int c0, int tpr, int sc, uint8_t* out0, int qpitch) {
  uint32_t k0[NW], k1[NW], k2[NW];
  const uint32_t* k = vkp + yy * 24;
#pragma unroll
  for (int j = 0; j < NW; ++j) {
    k0[j] = k[j];
    k1[j] = k[8 + j];
    k2[j] = k[16 + j];
  }
  const int f = vfirst[yy] - top;
  const uint32_t sel = 0x3210u + static_cast<uint32_t>(f & 3) * 0x1111u;
  uint8_t* out = out0 + yy * qpitch;
  for (int xx = c0; xx < sc; xx += tpr) {
    const uint32_t* wp = reinterpret_cast<const uint32_t*>(tmp + xx * rp + (f & ~3));
    uint32_t w[NW + 1];
#pragma unroll
    for (int j = 0; j <= NW; ++j) w[j] = wp[j];
    const int32_t v = window_sum<NW>(w, sel, k0, k1, k2) >> 22;
    out[xx] = static_cast<uint8_t>(v < 0 ? 0 : v > 255 ? 255 : v);
  }
}

// The source region a line's filter windows can reach into L2, a bulk prefetch a row (the copy
// engine streams it in from DRAM while the CTA works on the line before; no thread waits on it),
// each range rounded to 16 bytes inside the page's buffer.
__device__ __forceinline__ void prefetch_line(const CropParams& p, int line, int tid, int nthr) {
  const LineDesc L = p.lines[line];
  if (p.crops_in || L.wide >= 0) return;
  const PageDesc P = p.pages[L.page];
  const int H = p.height, cw = L.width;
  const double vsup = (L.y1 - L.y0) / H < 1.0 ? 1.0 : (L.y1 - L.y0) / H;
  const double hsup = (L.x1 - L.x0) / cw < 1.0 ? 1.0 : (L.x1 - L.x0) / cw;
  const int ylo = max(0, static_cast<int>(floor(L.y0 - vsup)) - 2), yhi = min(P.height, static_cast<int>(ceil(L.y1 + vsup)) + 2);
  const int xlo = max(0, static_cast<int>(floor(L.x0 - hsup)) - 2), xhi = min(P.width, static_cast<int>(ceil(L.x1 + hsup)) + 2);
  if (xhi <= xlo) return;
  const uintptr_t first = reinterpret_cast<uintptr_t>(P.data);
  const uintptr_t last = first + static_cast<uintptr_t>(static_cast<long long>(P.height - 1) * P.stride + P.width);
  for (int y = ylo + tid; y < yhi; y += nthr) {
    const uintptr_t row = first + static_cast<uintptr_t>(static_cast<long long>(y) * P.stride);
    uintptr_t a = (row + xlo) & ~uintptr_t(15), b = (row + xhi + 15) & ~uintptr_t(15);
    if (a < first) a += 16;
    if (b > last) b -= 16;
    if (b > a) l2_prefetch_bulk(reinterpret_cast<const void*>(a), static_cast<uint32_t>(b - a));
  }
}

// Persistent: a CTA takes lines one after another in p.order (its first is the blockIdx.x-th, the
// next ones claimed from p.claim[0] as it starts each line, so that the next line's region is
// prefetched while this one is worked on; the costliest lines first, so the last wave is short);
// the stem's constants and the tables are set up once a CTA.
template <bool kInt8>
__global__ void __launch_bounds__(kCropThreads, 2) crop_stem_kernel(const __grid_constant__ CropParams p) {
  extern __shared__ __align__(16) uint8_t sm[];
  __shared__ int s_next;
  const int H = p.height;
  const CropSmem S = crop_smem(H, p.max_bw);
  const int qpitch = S.qpitch;
  uint8_t* qb = sm + S.qb;
  uint8_t* tmp = sm + S.tmp;
  int32_t* hk = reinterpret_cast<int32_t*>(sm + S.hk);
  uint32_t* wq = reinterpret_cast<uint32_t*>(sm + S.wq);
  float* swf = reinterpret_cast<float*>(sm + S.swf);
  int32_t* soff = reinterpret_cast<int32_t*>(sm + S.soff);
  float* sscale = reinterpret_cast<float*>(sm + S.sscale);
  float* sbias = reinterpret_cast<float*>(sm + S.sbias);
  int32_t* vk = reinterpret_cast<int32_t*>(sm + S.vk);
  uint32_t* vkp = reinterpret_cast<uint32_t*>(sm + S.vkp);
  int32_t* vfirst = reinterpret_cast<int32_t*>(sm + S.vfirst);
  int32_t* vcount = reinterpret_cast<int32_t*>(sm + S.vcount);
  int32_t* hist = reinterpret_cast<int32_t*>(sm + S.hist);
  int32_t* red = reinterpret_cast<int32_t*>(sm + S.red);
  float* ftab = reinterpret_cast<float*>(sm + S.ftab);
  uint8_t* stab = sm + S.stab;
  const int tid = threadIdx.x, nthr = blockDim.x;
  const int taps_stem = p.kh * p.kw;
  auto px = [&](int y, int x) -> uint8_t& { return qb[(y + 2) * qpitch + x + 4]; };
  int claimed = blockIdx.x;
  if (claimed < p.n) prefetch_line(p, p.order[claimed], tid, nthr);

  // the stem's constants; INT8: a channel's taps as one word per kernel row (zeros past kw), and
  // the offset that turns the sum into kMagicBits + (sum - in_zero * colsum): |sum| <= 9 * 255 * 128
  if (kInt8) {
    for (int i = tid; i < kStemMaxOut * 3; i += nthr) {
      const int j = i / 3, ky = i % 3;
      uint32_t w = 0;
      if (j < p.cout && ky < p.kh)
        for (int kx = 0; kx < p.kw && kx < 4; ++kx)
          w |= static_cast<uint32_t>(static_cast<uint8_t>(p.w8[j * taps_stem + ky * p.kw + kx])) << (8 * kx);
      wq[i] = w;
    }
  } else {
    // [tap][channel]: a tap's weights for four channels are one 16-byte load (zeros past cout)
    for (int i = tid; i < kStemMaxOut * 9; i += nthr) {
      const int t = i / kStemMaxOut, j = i - t * kStemMaxOut;
      swf[i] = j < p.cout && t < taps_stem ? p.wf[j * taps_stem + t] : 0.0f;
    }
  }
  for (int i = tid; i < kStemMaxOut; i += nthr) {
    const bool in = i < p.cout;
    sscale[i] = kInt8 && in ? p.scale[i] : 1.0f;
    sbias[i] = in ? p.bias[i] : 0.0f;
    soff[i] = kInt8 && in ? kMagicBits - p.in_zero * p.colsum[i] : kMagicBits;
  }
  for (int i = tid; i < 256; i += nthr) {
    if (kInt8) stab[i] = p.in_table[i];
    // the FP16 engine's input: the ink 1 - p / 255 rounded to float16
    ftab[i] = __half2float(__float2half_rn(__fsub_rn(1.0f, __fdiv_rn(static_cast<float>(i), 255.0f))));
  }

  while (claimed < p.n) {
  const int line = p.order[claimed];
  if (tid == 0) s_next = static_cast<int>(gridDim.x) + atomicAdd(p.claim, 1);
  for (int i = tid; i < 256; i += nthr) hist[i] = 0;
  if (tid < 8) red[tid] = 0;
  // the tables and counters before any use (a ready crop goes straight to the final pass), the
  // claim; the line before is done with shared memory
  __syncthreads();
  const int next = s_next;
  if (next < p.n) prefetch_line(p, p.order[next], tid, nthr);
  const LineDesc L = p.lines[line];
  const PageDesc P = p.pages[L.page];
  const int bw = L.bw, cw = p.crops_in ? L.bw : L.width;

  bool flip = false;
  uint8_t ground = 0;
  if (!p.crops_in && L.wide >= 0) {
    // resampled by crop_wide_kernel: its raw crop into place
    const uint8_t* src = p.wide + static_cast<long long>(L.wide) * H * p.wide_pitch;
    for (int i = tid; i < H * cw; i += nthr) {
      const int y = i / cw, x = i - y * cw;
      px(y, x) = src[y * p.wide_pitch + x];
    }
  } else if (!p.crops_in) {
    // this line's tap stride (PIL's ksize), from a bound on the source rows the vertical windows
    // span (each window lies within [y0 - support - 1, y1 + support + 1]), and the taps a window
    // has at most: [floor(c - s + 0.5), floor(c + s + 0.5)) holds at most ceil(2 s) + 1 samples
    // (in words of 4 taps, the dp4a passes' unrolling, uniform over the line; the coefficient
    // setup checks every window against it)
    const double hscale = (L.x1 - L.x0) / cw, hsup = hscale < 1.0 ? 1.0 : hscale;
    const int T = min(kMaxTaps, static_cast<int>(ceil(hsup)) * 2 + 1);
    const double vspan = L.y1 - L.y0, vsup = vspan / H < 1.0 ? 1.0 : vspan / H;
    const int rows_ub = static_cast<int>(ceil(vspan + 2.0 * vsup)) + 4;
    const int nwh = (min(kMaxTaps, static_cast<int>(ceil(2.0 * hsup)) + 1) + 3) >> 2;
    const int nwv = (min(kMaxTaps, static_cast<int>(ceil(2.0 * vsup)) + 1) + 3) >> 2;
    // beyond this kernel's reach (the host sends such lines to crop_wide_kernel)
    if (static_cast<int>(ceil(vsup)) * 2 + 1 > kMaxTaps || static_cast<int>(ceil(hsup)) * 2 + 1 > kMaxTaps ||
        rows_ub > kMaxSrcRows) {
      if (tid == 0) atomicCAS(p.err, 0, kErrBadShape);
      break;
    }
    // the intermediate, column-major: a column of the strip holds its source rows contiguous in
    // rp bytes (the 8-row chunks, and the vertical windows' word reads, stay inside), rp / 4 odd
    // so that a warp's columns fall in distinct banks
    int rp = max((rows_ub + 7) & ~7, rows_ub + 4 * nwv + 4);
    rp = (rp + 3) & ~3;
    if (((rp >> 2) & 1) == 0) rp += 4;
    const int strip = max(16, min(kMaxStripCols, min(kStripBytes / rp, kCoefBytes / (4 * (T + 2)))));
    // horizontal coefficients (a thread a column) of `count` columns from x0: hk holds ncoef
    // columns' (at least a strip's; a line's whole width when it fits, so that the strips after
    // the first do not wait on the double-precision setup)
    const int ncoef = kCoefBytes / (4 * (T + 2));
    auto hcoeffs = [&](int x0, int count) {
      for (int xx = tid; xx < count; xx += nthr) {
        int32_t* c = hk + xx * (T + 2);
        int n;
        c[0] = coeffs(L.x0, L.x1, cw, x0 + xx, c + 2, &n, T);
        c[1] = n;
      }
    };
    // a window that does not fit the dp4a pass: more taps than the bound (or than kMaxHWords
    // words), or its word reads off the page
    auto hbad_of = [&](const int32_t* c) {
      return nwh > kMaxHWords || c[1] > 4 * nwh || c[0] < 0 || c[0] + 4 * nwh + 4 > P.width;
    };
    // vertical coefficients (rows from the last thread down, with their byte planes) and the
    // first block of horizontal ones (columns from thread 0 up)
    bool vbad_t = false;
    for (int yy = nthr - 1 - tid; yy < H; yy += nthr) {
      int n;
      int32_t* k = vk + yy * kMaxTaps;
      vfirst[yy] = coeffs(L.y0, L.y1, H, yy, k, &n);
      vcount[yy] = n;
      vbad_t |= n > 4 * nwv;
      uint32_t k0[8], k1[8], k2[8];
      weight_planes<8>(k, n, k0, k1, k2);
      uint32_t* kp = vkp + yy * 24;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        kp[j] = k0[j];
        kp[8 + j] = k1[j];
        kp[16 + j] = k2[j];
      }
    }
    hcoeffs(0, min(cw, ncoef));
    int xc0 = 0;  // the first column hk holds
    const bool vbad = __syncthreads_or(vbad_t) != 0;
    const int top = vfirst[0];
    const int rows = vfirst[H - 1] + vcount[H - 1] - top;
    if (rows > kMaxSrcRows || rows > rows_ub || strip * rp > kStripBytes) {
      if (tid == 0) atomicCAS(p.err, 0, kErrBadShape);
      break;
    }
    const int nchunks = (rows + 7) >> 3;
    const bool same_sel = (P.stride & 3) == 0;
    for (int x0 = 0; x0 < cw; x0 += strip) {
      const int sc = min(strip, cw - x0);
      if (x0 + sc > xc0 + ncoef) {
        __syncthreads();  // the previous strip's passes are done with hk
        xc0 = x0;
        hcoeffs(x0, min(cw - x0, ncoef));
        __syncthreads();
      }
      // a thread a column of the strip, the rows split into groups when the strip is narrow
      const int groups = max(1, nthr / sc);
      const int rg = tid / sc, xx = tid - rg * sc;
      const int32_t* c = hk + (x0 - xc0 + xx) * (T + 2);
      __syncthreads();  // the previous strip's vertical pass is done with tmp
      if (rg < groups) {
        // horizontal pass: every source row the vertical windows read, 8-row chunks split over
        // the row groups
        const int xmin = c[0], n = c[1];
        int32_t paper = 0;  // a row off the page: 255 * the weights' sum
        for (int t = 0; t < n; ++t) paper += 255 * c[2 + t];
        uint8_t* col = tmp + xx * rp;
        // a column's own choice (its row groups agree: same coefficients), so that a window at
        // the page's edge sends only its own column to the tap-by-tap loop below
        if (!hbad_of(c)) {
#define CREC_HPASS(NW)                                                                  \
  case NW:                                                                              \
    if (same_sel) hpass<NW, true>(P, c, paper, top, rg, nchunks, groups, col);          \
    else hpass<NW, false>(P, c, paper, top, rg, nchunks, groups, col);                  \
    break;
          switch (nwh) {
            CREC_HPASS(1)
            CREC_HPASS(2)
            CREC_HPASS(3)
            CREC_HPASS(4)
            CREC_HPASS(5)
          }
#undef CREC_HPASS
        } else {
          // a window off the page's edge (pixels there read as paper)
          for (int r = rg; r < rows; r += groups) {
            const int y = top + r;
            int32_t ss = 1 << 21;
            if (y >= 0 && y < P.height) {
              const uint8_t* src = P.data + static_cast<long long>(y) * P.stride + xmin;
              for (int t = 0; t < n; ++t) {
                const int x = xmin + t;
                ss += ((x >= 0 && x < P.width) ? static_cast<int32_t>(__ldg(src + t)) : 255) * c[2 + t];
              }
            } else {
              ss += paper;
            }
            col[r] = clip8d(ss);
          }
        }
      }
      __syncthreads();
      if (!vbad) {
        // vertical pass: the strip's output pixels, a thread a row and every tpr-th column
        const int tpr = nthr / H, yy = tid / tpr, c0 = tid - yy * tpr;
        if (yy < H) {
          uint8_t* out0 = &px(0, x0);
#define CREC_VPASS(NW) \
  case NW:             \
    vpass_rows<NW>(tmp, rp, vfirst, vkp, top, yy, c0, tpr, sc, out0, qpitch); \
    break;
          switch (nwv) {
            CREC_VPASS(1)
            CREC_VPASS(2)
            CREC_VPASS(3)
            CREC_VPASS(4)
            CREC_VPASS(5)
            CREC_VPASS(6)
            CREC_VPASS(7)
            CREC_VPASS(8)
          }
#undef CREC_VPASS
        }
      } else if (rg < groups) {
        const uint8_t* col = tmp + xx * rp;
        uint8_t* out = &px(0, x0 + xx);
        for (int yy = rg; yy < H; yy += groups) {
          const int f = vfirst[yy] - top, n = vcount[yy];
          const int32_t* k = vk + yy * kMaxTaps;
          int32_t ss = 1 << 21;
          for (int t = 0; t < n; ++t) ss += col[f + t] * k[t];
          out[yy * qpitch] = clip8d(ss);
        }
      }
    }
  }
  if (!p.crops_in) {
    __syncthreads();
    // finish: the ground's histogram (first row, last row, last column)
    for (int x = tid; x < cw; x += nthr) {
      atomicAdd(&hist[px(0, x)], 1);
      atomicAdd(&hist[px(H - 1, x)], 1);
    }
    for (int y = tid; y < H; y += nthr) atomicAdd(&hist[px(y, cw - 1)], 1);
    __syncthreads();
    const int count = 2 * cw + H;
    auto ground_of = [&](bool flipped) {
      return count % 2 ? hist_nth(hist, count / 2, flipped)
                       : (hist_nth(hist, count / 2 - 1, flipped) + hist_nth(hist, count / 2, flipped)) / 2;
    };
    if (tid < 32) {
      const int g = ground_of(false);
      if (tid == 0) red[0] = g;
    }
    __syncthreads();
    if (p.flip_margin > 0) {
      const int g = red[0], lo = g - p.flip_margin, hi = g + p.flip_margin;
      // four pixels a word (crop widths are multiples of 8, the crop starts at column 4 of qb):
      // byte-wise compares, their 0xff bytes counted by popc (8 bits a pixel); an item is a
      // (row, word), the quotient a multiply-high as in the final pass below
      int below = 0, above = 0, dark = 0;
      const int nw = cw >> 2;
      const uint32_t inv = static_cast<uint32_t>(0xffffffffu / static_cast<uint32_t>(nw)) + 1u;
      const uint32_t lo4 = static_cast<uint32_t>(lo < 0 ? 0 : lo) * 0x01010101u;
      const uint32_t hi4 = static_cast<uint32_t>(hi > 255 ? 255 : hi) * 0x01010101u;
      const bool any_lo = lo >= 0, any_hi = hi <= 255;
      for (int i = tid; i < H * nw; i += nthr) {
        const int y = static_cast<int>(__umulhi(static_cast<uint32_t>(i), inv)), w4 = i - y * nw;
        const uint32_t w = *reinterpret_cast<const uint32_t*>(&px(y, 4 * w4));
        if (any_lo) below += __popc(__vcmpleu4(w, lo4));
        if (any_hi) above += __popc(__vcmpgeu4(w, hi4));
        dark += __popc(__vcmpleu4(w, 0x7f7f7f7fu));
      }
      below >>= 3;
      above >>= 3;
      dark >>= 3;
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
    if (tid < 32) {
      const int g = ground_of(flip);
      if (tid == 0) red[4] = g;
    }
    __syncthreads();
    ground = static_cast<uint8_t>(red[4]);
  }
  // the finished crop (flipped, padded to the bucket width with the ground) and, for INT8, its
  // quantized input in place, the border the zero point; a thread a column of qb
  {
    const uint8_t* src = p.crops_in ? p.crops_in + static_cast<long long>(line) * H * p.crops_in_pitch : nullptr;
    uint8_t* dst = p.crops_out ? p.crops_out + static_cast<long long>(line) * H * p.crops_pitch : nullptr;
    const uint8_t zq = static_cast<uint8_t>(p.in_zero);
    if (!src && !dst) {
      // a thread a word (4 columns) of qb's rows: the flip a XOR, the INT8 input table a byte at
      // a time; words across the border, the pad or the crop's right edge byte by byte
      // item i: row i / wpr, word i % wpr (the quotient a multiply-high by 2^32 / wpr rounded up,
      // exact while i * wpr < 2^32)
      // only the words the stem reads: its windows' 8-byte reads start at most at qb column bw + 4
      // (at most 4 columns of left padding) and end before bw + 12, so bw / 4 + 3 words a row (5,
      // to spare); the rest of the run's widest row is never read for this line
      const int wpr = min(qpitch >> 2, (bw >> 2) + 5);
      const uint32_t inv = static_cast<uint32_t>(0xffffffffu / static_cast<uint32_t>(wpr)) + 1u;
      const uint32_t fx = flip ? 0xffffffffu : 0u;
      for (int i = tid; i < (H + 4) * wpr; i += nthr) {
        const int r = static_cast<int>(__umulhi(static_cast<uint32_t>(i), inv)), w4 = i - r * wpr;
        const int x0 = 4 * w4 - 4;
        {
          const int y = r - 2;
          uint32_t* qw = reinterpret_cast<uint32_t*>(qb + r * qpitch) + w4;
          if (y < 0 || y >= H || x0 + 3 < 0 || x0 >= bw) {
            if (kInt8) *qw = static_cast<uint32_t>(zq) * 0x01010101u;
            continue;
          }
          const uint32_t old = *qw;
          uint32_t v = 0;
          if (x0 >= 0 && x0 + 3 < cw) {
            const uint32_t f = old ^ fx;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint32_t b = (f >> (8 * k)) & 0xffu;
              v |= static_cast<uint32_t>(kInt8 ? stab[b] : b) << (8 * k);
            }
          } else {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const int x = x0 + k;
              uint32_t b;
              if (x < 0 || x >= bw) {
                b = kInt8 ? zq : (old >> (8 * k)) & 0xffu;
              } else {
                const uint32_t pix = x >= cw ? ground : ((old >> (8 * k)) & 0xffu) ^ (fx & 0xffu);
                b = kInt8 ? stab[pix] : pix;
              }
              v |= b << (8 * k);
            }
          }
          *qw = v;
        }
      }
    } else {
      // tests (the finished crops copied out) and crops given ready: a thread a column of qb
    for (int c = tid; c < qpitch; c += nthr) {
      const int x = c - 4;
      const bool col_in = x >= 0 && x < bw;
      for (int r = 0; r < H + 4; ++r) {
        const int y = r - 2;
        uint8_t& q = qb[r * qpitch + c];
        if (!col_in || y < 0 || y >= H) {
          if (kInt8) q = zq;
          continue;
        }
        uint8_t v;
        if (src) v = src[y * p.crops_in_pitch + x];
        else if (x >= cw) v = ground;
        else v = flip ? static_cast<uint8_t>(255 - q) : q;
        if (dst && x < p.crops_pitch) dst[y * p.crops_pitch + x] = v;
        q = kInt8 ? stab[v] : v;
      }
    }
    }
  }
  __syncthreads();

  // the stem, into the line's segment of the stem tensor: a thread two output pixels, (oy, ox) and
  // (oy + 1, ox), and all their channels; INT8: each weight and per-channel constant read from
  // shared memory serves both (the pixels' arithmetic is each its own, as for one pixel alone)
  const int oh = (H + 2 * p.pt - p.kh) / p.sh + 1, ow = (bw + 2 * p.pl - p.kw) / p.sw + 1;
  const int ph = (oh + 1) >> 1;  // pixel pairs down a column
  const long long col0 = static_cast<long long>(L.seg) >> p.out_shift;
  const int eb = kInt8 ? 1 : 2;
  const float lo = p.relu ? 0.0f : static_cast<float>(-p.out_zero), hi = static_cast<float>(255 - p.out_zero);
  const int32_t zc = p.out_zero - kMagicBits;
  const bool windows = kInt8 && p.kh <= 3 && p.kw <= 4 && p.pt >= 0 && p.pt <= 2 && p.pl >= 0 && p.pl <= 4;
  // pair i = tid + k * nthr as (pair row, ox), advanced without a division a step
  const int step_y = nthr / ow, step_x = nthr - step_y * ow;
  int py = tid / ow, ox = tid - py * ow;
  for (int i = tid; i < ph * ow; i += nthr, py += step_y, ox += step_x) {
    if (ox >= ow) {
      ox -= ow;
      ++py;
    }
    const int oy = 2 * py;
    const bool two = oy + 1 < oh;  // the pair's second pixel exists
    uint8_t* dst = p.out + (oy + p.out_ph) * p.out_pitch + (col0 + ox) * p.cp_out * eb;
    uint8_t* dst1 = dst + p.out_pitch;
    if constexpr (kInt8) {
      // a kernel row's taps, 4 bytes a word (past kw: anything, the weights there are 0); the
      // border reads the zero point: real zero
      uint32_t a[2][3] = {{0, 0, 0}, {0, 0, 0}};
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int y0 = oy + e;
        if (windows) {
          const int cs = ox * p.sw - p.pl + 4, rs = y0 * p.sh - p.pt + 2;
          const int al = cs & ~3;
          const uint32_t sel = 0x3210u + static_cast<uint32_t>(cs & 3) * 0x1111u;
#pragma unroll
          for (int ky = 0; ky < 3; ++ky) {
            if (ky < p.kh && (e == 0 || two)) {
              const uint8_t* rp = qb + (rs + ky) * qpitch + al;
              a[e][ky] = __byte_perm(*reinterpret_cast<const uint32_t*>(rp), *reinterpret_cast<const uint32_t*>(rp + 4), sel);
            }
          }
        } else if (e == 0 || two) {
          for (int ky = 0; ky < p.kh && ky < 3; ++ky)
            for (int kx = 0; kx < p.kw && kx < 4; ++kx) {
              const int y = y0 * p.sh - p.pt + ky, x = ox * p.sw - p.pl + kx;
              const uint32_t q = (y >= 0 && y < H && x >= 0 && x < bw) ? px(y, x) : static_cast<uint32_t>(p.in_zero);
              a[e][ky] |= q << (8 * kx);
            }
        }
      }
      // sum over taps of (a - zero) * w = dp4a(a, w) - zero * colsum, exact in int32; then the
      // output stage with exact conversions (kMagic), rounded before the clamp where the host's
      // bound allows (the clamp is then the saturating byte pack)
      auto channels = [&](auto round_first) {
      constexpr bool kRound = decltype(round_first)::value;
      for (int c16 = 0; c16 < p.cp_out; c16 += 16) {
        uint32_t wv[2][4];
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          const int j = c16 + 4 * c4;
          const uint4* w4 = reinterpret_cast<const uint4*>(wq + j * 3);
          const uint4 wa = w4[0], wb = w4[1], wc = w4[2];
          const uint32_t w[12] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w, wc.x, wc.y, wc.z, wc.w};
          const int4 o4 = *reinterpret_cast<const int4*>(soff + j);
          const float4 s4 = *reinterpret_cast<const float4*>(sscale + j);
          const float4 b4 = *reinterpret_cast<const float4*>(sbias + j);
          const int32_t oo[4] = {o4.x, o4.y, o4.z, o4.w};
          const float ss[4] = {s4.x, s4.y, s4.z, s4.w}, bb[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            int32_t code[4], acc[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              acc[u] = dp4a_us(a[e][0], w[3 * u], oo[u]);
              acc[u] = dp4a_us(a[e][1], w[3 * u + 1], acc[u]);
              acc[u] = dp4a_us(a[e][2], w[3 * u + 2], acc[u]);
            }
#pragma unroll
            for (int u = 0; u < 4; u += 2) {  // two channels at a time on the packed FP32 pipe
              float2 q = out_stage2(acc[u], acc[u + 1], make_float2(ss[u], ss[u + 1]), make_float2(bb[u], bb[u + 1]),
                                    p.out_inv_scale);
              if (!kRound) {
                q.x = fminf(fmaxf(q.x, lo), hi);
                q.y = fminf(fmaxf(q.y, lo), hi);
              }
              int32_t t0, t1;
              magic_rint_bits2(q, t0, t1);
              code[u] = t0 + zc;
              code[u + 1] = t1 + zc;
            }
            wv[e][c4] = pack_sat_u8x4(code);
          }
        }
        *reinterpret_cast<uint4*>(dst + c16) = make_uint4(wv[0][0], wv[0][1], wv[0][2], wv[0][3]);
        if (two) *reinterpret_cast<uint4*>(dst1 + c16) = make_uint4(wv[1][0], wv[1][1], wv[1][2], wv[1][3]);
      }
      };
      if (p.sat) channels(std::true_type{});
      else channels(std::false_type{});
    } else {
      // each pixel of the pair on its own: 16 channels as 8 pairs, an fma chain over the taps in tap
      // order from 0 on the packed FP32 pipe (the FP16 engine is graded by tolerance), + bias,
      // ReLU, to FP16 (pairing the pixels as INT8 does was slower here: more registers, narrower stores)
      for (int e = 0; e < (two ? 2 : 1); ++e) {
        float in[9];
#pragma unroll
        for (int t = 0; t < 9; ++t) {
          in[t] = 0.0f;
          if (t >= taps_stem) continue;
          const int y = (oy + e) * p.sh - p.pt + t / p.kw, x = ox * p.sw - p.pl + t % p.kw;
          if (y < 0 || y >= H || x < 0 || x >= bw) continue;  // the border: real zero
          in[t] = ftab[px(y, x)];
        }
        uint8_t* d = e ? dst1 : dst;
        for (int c0 = 0; c0 < p.cp_out; c0 += 16) {
          float2 acc[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) acc[q] = make_float2(0.0f, 0.0f);
#pragma unroll
          for (int t = 0; t < 9; ++t) {
            if (t >= taps_stem) break;
            const float2 x2 = make_float2(in[t], in[t]);
            const float4* w4 = reinterpret_cast<const float4*>(swf + t * kStemMaxOut + c0);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const float4 w = w4[k];
              acc[2 * k] = __ffma2_rn(x2, make_float2(w.x, w.y), acc[2 * k]);
              acc[2 * k + 1] = __ffma2_rn(x2, make_float2(w.z, w.w), acc[2 * k + 1]);
            }
          }
          alignas(16) __half2 o[8];
          const float4* b4 = reinterpret_cast<const float4*>(sbias + c0);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float4 b = b4[k];
            float v[4] = {__fadd_rn(acc[2 * k].x, b.x), __fadd_rn(acc[2 * k].y, b.y), __fadd_rn(acc[2 * k + 1].x, b.z),
                          __fadd_rn(acc[2 * k + 1].y, b.w)};
            if (p.relu) {
#pragma unroll
              for (int u = 0; u < 4; ++u) v[u] = v[u] > 0.0f ? v[u] : 0.0f;
            }
            o[2 * k] = __floats2half2_rn(v[0], v[1]);
            o[2 * k + 1] = __floats2half2_rn(v[2], v[3]);
          }
          *reinterpret_cast<uint4*>(d + c0 * 2) = *reinterpret_cast<const uint4*>(o);
          *reinterpret_cast<uint4*>(d + c0 * 2 + 16) = *reinterpret_cast<const uint4*>(o + 4);
        }
      }
    }
  }
  // the gap after this line's segment (and before the first line's), the zero point
  const long long gap0 = col0 + ow, gap1 = static_cast<long long>(L.next_seg) >> p.out_shift;
  const int lead = line == 0 ? static_cast<int>(col0) : 0;
  const int gapn = static_cast<int>(gap1 - gap0) + lead;
  const int vec = p.cp_out * eb / 16;
  const uint32_t zb = kInt8 ? static_cast<uint32_t>(p.out_zero) * 0x01010101u : 0u;
  const uint4 z4 = make_uint4(zb, zb, zb, zb);
  for (int i = tid; i < gapn * oh * vec; i += nthr) {
    const int v = i % vec, rest = i / vec;
    const int c = rest % gapn, oy = rest / gapn;
    const long long col = c < lead ? c : gap0 + (c - lead);
    *reinterpret_cast<uint4*>(p.out + (oy + p.out_ph) * p.out_pitch + col * p.cp_out * eb + v * 16) = z4;
  }
  claimed = next;
  }
  // the claim counters back to 0 for the next launch, by the last CTA out (every claim is made by
  // then: a CTA counts itself out after its last claim)
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(p.claim + 1, 1) == static_cast<int>(gridDim.x) - 1) {
      p.claim[0] = 0;
      p.claim[1] = 0;
    }
  }
}

// Shared memory of crop_wide_kernel: vertical coefficients [height][vtaps], their first rows and
// counts, a strip's horizontal coefficients [hk_cols][htaps + 2] (first, count, taps), the
// intermediate [rows][strip columns].
__host__ __device__ inline size_t wide_smem(int height, int vtaps, int htaps, int hk_cols, int tmp_bytes) {
  return static_cast<size_t>(height) * (vtaps + 2) * 4 + static_cast<size_t>(hk_cols) * (htaps + 2) * 4 +
         static_cast<size_t>(tmp_bytes);
}

// The resampling of a line beyond crop_stem_kernel's reach (downscales past 15x, or more source
// rows than kMaxSrcRows), one CTA a line, the scalar passes of carbon/src/lines.cpp:117-147
// (resample_scalar): the same coefficients (coeffs), the horizontal pass over every source row
// the vertical windows span into an 8-bit intermediate, a strip of columns at a time, then the
// vertical pass.  Writes the raw crop (not yet finished) to out[slot]; crop_stem_kernel finishes it.
__global__ void __launch_bounds__(kCropThreads) crop_wide_kernel(const __grid_constant__ WideParams p) {
  extern __shared__ __align__(16) uint8_t sm[];
  const int slot = blockIdx.x;
  const LineDesc L = p.lines[p.index[slot]];
  const PageDesc P = p.pages[L.page];
  const int H = p.height, cw = L.width;
  int32_t* vk = reinterpret_cast<int32_t*>(sm);
  int32_t* vfirst = vk + H * p.vtaps;
  int32_t* vcount = vfirst + H;
  int32_t* hk = vcount + H;
  const int hstride = p.htaps + 2;
  uint8_t* tmp = reinterpret_cast<uint8_t*>(hk + p.hk_cols * hstride);
  const int tid = threadIdx.x, nthr = blockDim.x;
  // the line's ksize each way against the buffers' (uniform over the CTA)
  const double hscale = (L.x1 - L.x0) / cw, hsup = hscale < 1.0 ? 1.0 : hscale;
  const double vscale = (L.y1 - L.y0) / H, vsup = vscale < 1.0 ? 1.0 : vscale;
  if (static_cast<int>(ceil(hsup)) * 2 + 1 > p.htaps || static_cast<int>(ceil(vsup)) * 2 + 1 > p.vtaps) {
    if (tid == 0) atomicCAS(p.err, 0, kErrBadShape);
    return;
  }
  for (int yy = tid; yy < H; yy += nthr) {
    int n;
    vfirst[yy] = coeffs(L.y0, L.y1, H, yy, vk + yy * p.vtaps, &n, p.vtaps);
    vcount[yy] = n;
  }
  __syncthreads();
  const int top = vfirst[0], rows = vfirst[H - 1] + vcount[H - 1] - top;
  if (rows <= 0 || rows > p.tmp_bytes) {
    if (tid == 0) atomicCAS(p.err, 0, kErrBadShape);
    return;
  }
  const int strip = min(p.hk_cols, p.tmp_bytes / rows);
  uint8_t* out = p.out + static_cast<long long>(slot) * H * p.pitch;
  for (int x0 = 0; x0 < cw; x0 += strip) {
    const int sc = min(strip, cw - x0);
    for (int xx = tid; xx < sc; xx += nthr) {
      int32_t* c = hk + xx * hstride;
      int n;
      c[0] = coeffs(L.x0, L.x1, cw, x0 + xx, c + 2, &n, p.htaps);
      c[1] = n;
    }
    __syncthreads();
    // horizontal: item (r, xx), the columns of a row side by side; pixels off the page read as paper
    for (int i = tid; i < rows * sc; i += nthr) {
      const int r = i / sc, xx = i - r * sc;
      const int32_t* c = hk + xx * hstride;
      const int xmin = c[0], n = c[1], y = top + r;
      int32_t ss = 1 << 21;
      if (y >= 0 && y < P.height) {
        const uint8_t* src = P.data + static_cast<long long>(y) * P.stride;
        for (int t = 0; t < n; ++t) {
          const int x = xmin + t;
          ss += ((x >= 0 && x < P.width) ? static_cast<int32_t>(__ldg(src + x)) : 255) * c[2 + t];
        }
      } else {
        for (int t = 0; t < n; ++t) ss += 255 * c[2 + t];
      }
      tmp[i] = clip8d(ss);
    }
    __syncthreads();
    // vertical: item (yy, xx)
    for (int i = tid; i < H * sc; i += nthr) {
      const int yy = i / sc, xx = i - yy * sc;
      const int f = vfirst[yy] - top, n = vcount[yy];
      const int32_t* k = vk + yy * p.vtaps;
      int32_t ss = 1 << 21;
      for (int t = 0; t < n; ++t) ss += static_cast<int32_t>(tmp[(f + t) * sc + xx]) * k[t];
      out[yy * p.pitch + x0 + xx] = clip8d(ss);
    }
    __syncthreads();  // the strip's intermediate and coefficients before the next strip's
  }
}

}  // namespace crec
