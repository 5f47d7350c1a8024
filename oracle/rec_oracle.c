/* A CPU restatement, in plain C, of the reference's line-recognition path: the
 * crop rule, the native executor's int8 and FP32 arithmetic on a recognizer, and
 * greedy CTC decoding.
 *
 * TEST INFRASTRUCTURE ONLY.  This is the parity checker for the CUDA path: only
 * tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load it.  It is
 * pinned against the reference's own compiled code (oracle/_ref) and against the
 * golden values of the reference's tests (tests/ in this repository).
 *
 * Each function cites the reference code it restates (paths within the reference
 * project).  Build: gcc -O2 -std=c11 -ffp-contract=off -fPIC -shared (contraction
 * off, as the reference builds its CPU code, so every double and float operation
 * rounds on its own).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------ crop rule */

typedef struct {
  int height, width_step, frame_px;
  double pad_v, pad_h;
  int flip_margin, flip_needs_dark;
} orc_rule;

ORC_API void orc_default_rule(orc_rule* r) {
  r->height = 32;
  r->width_step = 8;
  r->frame_px = 4;
  r->pad_v = 0.2;
  r->pad_h = 0.3;
  r->flip_margin = 48;
  r->flip_needs_dark = 1;
}

/* carbon/src/lines.cpp:33-44 (crop_region): the same expressions in the same order. */
ORC_API int orc_crop_region(const double* b, const orc_rule* r, double* region) {
  const double h = b[3] - b[1];
  const double sy0 = b[1] - r->pad_v * h, sy1 = b[3] + r->pad_v * h;
  const double scale = r->height / (sy1 - sy0);
  const double w_src = (b[2] - b[0]) + 2 * r->pad_h * h;
  int width = (int)ceil(w_src * scale / r->width_step - 1e-6) * r->width_step;
  if (width < r->width_step) width = r->width_step;
  const double extra = (width / scale - w_src) / 2;
  region[0] = b[0] - r->pad_h * h - extra;
  region[1] = sy0;
  region[2] = b[2] + r->pad_h * h + extra;
  region[3] = sy1;
  return width;
}

/* carbon/src/engine.cpp:669-675 (width_bucket): the ladder from 32 by x1.3, multiples of 8, to 2048. */
ORC_API int orc_width_bucket(int w) {
  for (int b = 32;;) {
    if (w <= b) return b;
    if (b >= 2048) return (w + 7) / 8 * 8;
    int nb = (int)ceil(b * 1.3);
    nb = (nb + 7) / 8 * 8;
    b = nb < 2048 ? nb : 2048;
  }
}

/* carbon/src/resample_math.h:32-77: PIL's bilinear precompute in double, 22-bit fixed point. */
#define PREC_BITS 22
static double triangle(double x) {
  if (x < 0.0) x = -x;
  return x < 1.0 ? 1.0 - x : 0.0;
}
static int floor_int(double v) {
  const int i = (int)v;
  return i - (v < i ? 1 : 0);
}
typedef struct {
  double scale, support, ss;
} filt;
static filt filter_for(double in0, double in1, int out) {
  filt f;
  f.scale = (in1 - in0) / out;
  const double fs = f.scale < 1.0 ? 1.0 : f.scale;
  f.support = 1.0 * fs;
  f.ss = 1.0 / fs;
  return f;
}
static int max_taps(filt f) { return (int)ceil(f.support) * 2 + 1; }
static int coefficients(filt f, double in0, int xx, int32_t* k, int* count) {
  const double center = in0 + (xx + 0.5) * f.scale;
  const int xmin = floor_int(center - f.support + 0.5);
  const int n = floor_int(center + f.support + 0.5) - xmin;
  double ww = 0.0;
  for (int x = 0; x < n; ++x) ww += triangle((x + xmin - center + 0.5) * f.ss);
  for (int x = 0; x < n; ++x) {
    double w = triangle((x + xmin - center + 0.5) * f.ss);
    if (ww != 0.0) w /= ww;
    k[x] = (int32_t)(w < 0 ? -0.5 + w * (1 << PREC_BITS) : 0.5 + w * (1 << PREC_BITS));
  }
  *count = n;
  return xmin;
}
static uint8_t clip8(int32_t v) {
  v >>= PREC_BITS;
  return (uint8_t)(v < 0 ? 0 : v > 255 ? 255 : v);
}

/* carbon/src/lines.cpp:119-160 (resample_scalar, the reference the vector passes equal):
 * horizontal pass over every row the vertical one reads into an 8-bit intermediate, then
 * the vertical pass; pixels off the image are paper (255). */
ORC_API int orc_resample_gray(const uint8_t* im, int iw, int ih, int64_t stride, double x0, double y0, double x1,
                              double y1, int ow, int oh, uint8_t* out, int64_t os) {
  if (ow <= 0 || oh <= 0) return -1;
  const filt fx = filter_for(x0, x1, ow), fy = filter_for(y0, y1, oh);
  const int tx = max_taps(fx), ty = max_taps(fy);
  int32_t* kx = (int32_t*)calloc((size_t)ow * tx, 4);
  int32_t* ky = (int32_t*)calloc((size_t)oh * ty, 4);
  int* fxs = (int*)malloc(sizeof(int) * ow * 2);
  int* fys = (int*)malloc(sizeof(int) * oh * 2);
  for (int i = 0; i < ow; ++i) fxs[2 * i] = coefficients(fx, x0, i, kx + (size_t)i * tx, &fxs[2 * i + 1]);
  for (int i = 0; i < oh; ++i) fys[2 * i] = coefficients(fy, y0, i, ky + (size_t)i * ty, &fys[2 * i + 1]);
  const int top = fys[0];
  const int rows = fys[2 * (oh - 1)] + fys[2 * (oh - 1) + 1] - top;
  uint8_t* tmp = (uint8_t*)malloc((size_t)(rows > 0 ? rows : 1) * ow);
  for (int r = 0; r < rows; ++r) {
    const int y = top + r;
    const uint8_t* row = (y >= 0 && y < ih) ? im + (int64_t)y * stride : NULL;
    for (int xx = 0; xx < ow; ++xx) {
      const int32_t* k = kx + (size_t)xx * tx;
      const int xmin = fxs[2 * xx], n = fxs[2 * xx + 1];
      int32_t ss = 1 << (PREC_BITS - 1);
      for (int i = 0; i < n; ++i) {
        const int x = xmin + i;
        const int v = (row && x >= 0 && x < iw) ? row[x] : 255;
        ss += v * k[i];
      }
      tmp[(size_t)r * ow + xx] = clip8(ss);
    }
  }
  for (int yy = 0; yy < oh; ++yy) {
    const int32_t* k = ky + (size_t)yy * ty;
    const uint8_t* src = tmp + (size_t)(fys[2 * yy] - top) * ow;
    const int n = fys[2 * yy + 1];
    for (int xx = 0; xx < ow; ++xx) {
      int32_t ss = 1 << (PREC_BITS - 1);
      for (int i = 0; i < n; ++i) ss += src[(size_t)i * ow + xx] * k[i];
      out[(int64_t)yy * os + xx] = clip8(ss);
    }
  }
  free(kx);
  free(ky);
  free(fxs);
  free(fys);
  free(tmp);
  return 0;
}

/* carbon/src/lines.cpp:249-270 (ground_histogram, ground_of): the median of the first row,
 * the last row and the last column (corners twice), an even count's two middle values
 * averaged and rounded down; of the flipped crop, read backwards. */
static void ground_histogram(const uint8_t* c, int w, int h, int64_t stride, int* hist) {
  memset(hist, 0, 256 * sizeof(int));
  for (int x = 0; x < w; ++x) {
    ++hist[c[x]];
    ++hist[c[(int64_t)(h - 1) * stride + x]];
  }
  for (int y = 0; y < h; ++y) ++hist[c[(int64_t)y * stride + w - 1]];
}
static int nth_of(const int* hist, int n, int flipped) {
  for (int v = 0, seen = 0; v < 256; ++v) {
    seen += hist[flipped ? 255 - v : v];
    if (seen > n) return v;
  }
  return 255;
}
static uint8_t ground_of(const int* hist, int count, int flipped) {
  return (uint8_t)(count % 2 ? nth_of(hist, count / 2, flipped)
                             : (nth_of(hist, count / 2 - 1, flipped) + nth_of(hist, count / 2, flipped)) / 2);
}
ORC_API int orc_crop_ground(const uint8_t* c, int w, int h, int64_t stride) {
  int hist[256];
  ground_histogram(c, w, h, stride, hist);
  return ground_of(hist, 2 * w + h, 0);
}

/* carbon/src/cpu/kernels.cpp:780-797 (count_beyond, the reference loop). */
static void count_beyond(const uint8_t* c, int w, int h, int64_t stride, int lo, int hi, int64_t* below,
                         int64_t* above) {
  *below = *above = 0;
  for (int y = 0; y < h; ++y) {
    const uint8_t* row = c + (int64_t)y * stride;
    for (int x = 0; x < w; ++x) {
      *below += row[x] <= lo;
      *above += row[x] >= hi;
    }
  }
}

/* carbon/src/lines.cpp:311-329 (finish_crop): flipped (255 - v) if light on dark (more bytes
 * at least flip_margin above the ground than below it; with flip_needs_dark also over half
 * the bytes at most 127), then padded to out_width with the (flipped) ground. */
ORC_API void orc_finish_crop(uint8_t* c, int w, int out_width, const orc_rule* r) {
  const int h = r->height;
  if (w <= 0 || h <= 0) return;
  int hist[256];
  ground_histogram(c, w, h, out_width, hist);
  int flip = 0;
  if (r->flip_margin > 0) {
    const int g = ground_of(hist, 2 * w + h, 0);
    int64_t below, above;
    count_beyond(c, w, h, out_width, g - r->flip_margin, g + r->flip_margin, &below, &above);
    flip = above > below;
  }
  if (flip && r->flip_needs_dark) {
    int64_t below, above;
    count_beyond(c, w, h, out_width, 127, 256, &below, &above);
    flip = 2 * below > (int64_t)w * h;
  }
  if (flip) {
    for (int y = 0; y < h; ++y)
      for (int x = 0; x < w; ++x) c[y * out_width + x] = (uint8_t)(255 - c[y * out_width + x]);
  }
  if (w < out_width) {
    const uint8_t g = ground_of(hist, 2 * w + h, flip);
    for (int y = 0; y < h; ++y) memset(c + (int64_t)y * out_width + w, g, (size_t)(out_width - w));
  }
}

/* carbon/src/lines.cpp:279-297 (crop_lines): each box's region resampled to its own width,
 * then finished at the batch width.  Returns -2 (and touches nothing after) if a crop is
 * wider than out_width. */
ORC_API int orc_crop_lines(const uint8_t* page, int w, int h, int64_t stride, const double* boxes, int n,
                           int out_width, uint8_t* out, int32_t* widths, const orc_rule* r) {
  const size_t plane = (size_t)r->height * out_width;
  for (int i = 0; i < n; ++i) {
    double reg[4];
    const int cw = orc_crop_region(boxes + 4 * i, r, reg);
    if (cw > out_width) return -2;
    uint8_t* o = out + (size_t)i * plane;
    orc_resample_gray(page, w, h, stride, reg[0], reg[1], reg[2], reg[3], cw, r->height, o, out_width);
    orc_finish_crop(o, cw, out_width, r);
    widths[i] = cw;
  }
  return 0;
}

/* ------------------------------------------------------------------ the recognizer */

/* The model blob written by carbon_rec/netdef.py (RecNet.to_blob). */
typedef struct {
  int c, u8, ph, pw;
  float scale;
  int zero;
} orc_value;

typedef struct {
  int kind, in, out, residual;
  int kh, kw, sh, sw, pt, pl, pb, pr, cin, cout, relu, fh, fw, res_fh, res_shift, int8;
  int8_t* w8;   /* [cout][cin/g][kh][kw] */
  float* wf;    /* same, float */
  float* wsc;   /* [cout] weight scales */
  float* bias;  /* [cout] */
  float* scale; /* [cout]: the sums' scale, the input's scale times the weights' (net.cpp:703) */
  int32_t* wt;  /* int8 weights as [tap][cin][cout] for the loops below */
  float* wtf;   /* float weights as [tap][cin][cout] */
} orc_layer;

typedef struct {
  int quantized, nv, nl, inp, outv, height;
  orc_value* v;
  orc_layer* l;
} orc_model;

static uint32_t rd32(const uint8_t** p) {
  uint32_t v;
  memcpy(&v, *p, 4);
  *p += 4;
  return v;
}

ORC_API void orc_model_close(void* h) {
  orc_model* m = (orc_model*)h;
  if (!m) return;
  for (int i = 0; i < m->nl; ++i) {
    free(m->l[i].w8);
    free(m->l[i].wf);
    free(m->l[i].wsc);
    free(m->l[i].bias);
    free(m->l[i].scale);
    free(m->l[i].wt);
    free(m->l[i].wtf);
  }
  free(m->l);
  free(m->v);
  free(m);
}

ORC_API void* orc_model_open(const uint8_t* blob, size_t len) {
  if (len < 40 || memcmp(blob, "CRECMDL1", 8) != 0) return NULL;
  const uint8_t* p = blob + 8;
  if (rd32(&p) != 1) return NULL;
  orc_model* m = (orc_model*)calloc(1, sizeof *m);
  m->quantized = rd32(&p) == 0;
  m->nv = (int)rd32(&p);
  m->nl = (int)rd32(&p);
  m->inp = (int)rd32(&p);
  m->outv = (int)rd32(&p);
  m->height = (int)rd32(&p);
  rd32(&p);
  m->v = (orc_value*)calloc((size_t)m->nv, sizeof(orc_value));
  m->l = (orc_layer*)calloc((size_t)m->nl, sizeof(orc_layer));
  for (int i = 0; i < m->nv; ++i) {
    orc_value* v = &m->v[i];
    v->c = (int)rd32(&p);
    v->u8 = (int)rd32(&p);
    memcpy(&v->scale, p, 4);
    p += 4;
    v->zero = (int)rd32(&p);
    v->ph = (int)rd32(&p);
    v->pw = (int)rd32(&p);
  }
  for (int i = 0; i < m->nl; ++i) {
    orc_layer* l = &m->l[i];
    int* f = &l->kind;
    for (int k = 0; k < 4; ++k) f[k] = (int)rd32(&p);
    int* g = &l->kh;
    for (int k = 0; k < 16; ++k) g[k] = (int)rd32(&p);
    if (l->kind == 2) continue;
    const int groups = l->kind == 1 ? l->cin : 1;
    const int taps = l->kh * l->kw, cpg = l->cin / groups;
    const size_t nw = (size_t)l->cout * cpg * taps;
    if (l->int8) {
      l->w8 = (int8_t*)malloc(nw);
      memcpy(l->w8, p, nw);
      p += (nw + 3) / 4 * 4;
      l->wsc = (float*)malloc(4 * (size_t)l->cout);
      memcpy(l->wsc, p, 4 * (size_t)l->cout);
      p += 4 * (size_t)l->cout;
      l->scale = (float*)malloc(4 * (size_t)l->cout);
      for (int j = 0; j < l->cout; ++j) l->scale[j] = m->v[l->in].scale * l->wsc[j];
      l->wt = (int32_t*)malloc(4 * nw);
      for (int j = 0; j < l->cout; ++j)
        for (int c = 0; c < cpg; ++c)
          for (int t = 0; t < taps; ++t) l->wt[((size_t)t * cpg + c) * l->cout + j] = l->w8[((size_t)j * cpg + c) * taps + t];
    } else {
      l->wf = (float*)malloc(4 * nw);
      memcpy(l->wf, p, 4 * nw);
      p += 4 * nw;
      l->wtf = (float*)malloc(4 * nw);
      for (int j = 0; j < l->cout; ++j)
        for (int c = 0; c < cpg; ++c)
          for (int t = 0; t < taps; ++t) l->wtf[((size_t)t * cpg + c) * l->cout + j] = l->wf[((size_t)j * cpg + c) * taps + t];
    }
    l->bias = (float*)malloc(4 * (size_t)l->cout);
    memcpy(l->bias, p, 4 * (size_t)l->cout);
    p += 4 * (size_t)l->cout;
  }
  if ((size_t)(p - blob) != len) {
    orc_model_close(m);
    return NULL;
  }
  return m;
}

ORC_API int orc_model_classes(void* h) {
  orc_model* m = (orc_model*)h;
  return m->v[m->outv].c;
}

/* carbon/src/net/net.cpp:84-90 (quantize): v / scale, clamped to +-2^22, rounded half to even
 * by adding and taking away 1.5 * 2^23, plus the zero point, clamped to 0..255. */
static uint8_t quantize_in(float v, float scale, int zero) {
  float r = v / scale;
  r = r < -4194304.0f ? -4194304.0f : r;
  r = r > 4194304.0f ? 4194304.0f : r;
  volatile float t = r + 12582912.0f; /* volatile: the two roundings happen as written */
  r = t - 12582912.0f;
  r += (float)zero;
  r = r > 255.0f ? 255.0f : r;
  r = r < 0.0f ? 0.0f : r;
  return (uint8_t)r;
}

/* The input table: a crop byte p becomes the ink 1 - p / 255 (carbon/src/pipeline.cpp:153),
 * quantized as the graph's input (net.cpp:250-262). */
ORC_API void orc_input_table(void* h, uint8_t* table) {
  orc_model* m = (orc_model*)h;
  const orc_value* x = &m->v[m->inp];
  for (int p = 0; p < 256; ++p) table[p] = quantize_in(1.0f - (float)p / 255.0f, x->scale, x->zero);
}

/* A tensor: NHWC for n lines, h x w, with a border of ph rows and pw columns holding the zero
 * point (uint8) or 0 (float), as the reference keeps them (net.cpp:100-160). */
typedef struct {
  int n, h, w, c, ph, pw;
  uint8_t* b;
  float* f;
} tens;
static int64_t tpix(const tens* t, int i, int y, int x) {
  return (((int64_t)i * (t->h + 2 * t->ph) + y + t->ph) * (t->w + 2 * t->pw) + x + t->pw) * t->c;
}
static void tens_alloc(tens* t, const orc_value* v, int u8, int n, int h, int w) {
  t->n = n;
  t->h = h;
  t->w = w;
  t->c = v->c;
  t->ph = v->ph;
  t->pw = v->pw;
  const size_t size = (size_t)n * (h + 2 * v->ph) * (w + 2 * v->pw) * v->c;
  if (u8) {
    t->b = (uint8_t*)malloc(size);
    memset(t->b, v->zero, size);
    t->f = NULL;
  } else {
    t->f = (float*)calloc(size, 4);
    t->b = NULL;
  }
}

/* carbon/src/cpu/kernels.h:354-380 (epilogue_scalar) for one output value: the int8 sum times
 * its scale, plus the bias, plus the residual (uint8 dequantized), ReLU, then requantized:
 * times the inverse scale, clamped to [-zero, 255 - zero], rounded half to even, plus zero. */
static float epi_float(float v, const orc_layer* l, int j, const tens* r, const orc_value* rv, int64_t ri) {
  if (l->int8) v = v * l->scale[j];
  v = v + l->bias[j];
  if (r) {
    if (r->b) {
      v = v + (float)((int32_t)r->b[ri] - rv->zero) * rv->scale;
    } else {
      v = v + r->f[ri];
    }
  }
  if (l->relu) v = v > 0 ? v : 0.0f;
  return v;
}
static uint8_t requant(float v, const orc_value* o) {
  const float lo = (float)(-o->zero), hi = (float)(255 - o->zero);
  const float inv = 1.0f / o->scale;
  float q = v * inv;
  q = q > lo ? q : lo;
  q = q < hi ? q : hi;
  return (uint8_t)((int32_t)nearbyintf(q) + o->zero);
}

/* One layer.  Dense and depthwise convolutions: int8 sums of (a - zero) * w
 * (carbon/src/cpu/kernels.cpp:140-154, 184-194) or FP32 FMA chains in the order of the taps then
 * the channels (:156-170, :172-182); the residual at row i >> shift (an upsampling read in
 * place).  Resize: nearest, whole scales, bytes copied (net.cpp:819-851). */
static void run_layer(const orc_model* m, const orc_layer* l, tens* vals) {
  const tens* x = &vals[l->in];
  tens* y = &vals[l->out];
  const orc_value* ov = &m->v[l->out];
  const int u8 = m->quantized && ov->u8;
  if (l->kind == 2) {
    tens_alloc(y, ov, u8, x->n, x->h * l->fh, x->w * l->fw);
    for (int i = 0; i < y->n; ++i)
      for (int oy = 0; oy < y->h; ++oy)
        for (int ox = 0; ox < y->w; ++ox) {
          const int64_t s = tpix(x, i, oy / l->fh, ox / l->fw), d = tpix(y, i, oy, ox);
          if (u8)
            memcpy(y->b + d, x->b + s, (size_t)y->c);
          else
            memcpy(y->f + d, x->f + s, sizeof(float) * y->c);
        }
    return;
  }
  const int oh = (x->h + l->pt + l->pb - l->kh) / l->sh + 1, ow = (x->w + l->pl + l->pr - l->kw) / l->sw + 1;
  tens_alloc(y, ov, u8, x->n, oh, ow);
  const int taps = l->kh * l->kw, dw = l->kind == 1;
  const int cpg = dw ? 1 : l->cin;
  const tens* r = l->residual >= 0 ? &vals[l->residual] : NULL;
  const orc_value* rv = l->residual >= 0 ? &m->v[l->residual] : NULL;
  const orc_value* xv = &m->v[l->in];
  int32_t* si = (int32_t*)malloc(4 * (size_t)l->cout);
  float* sf = (float*)malloc(4 * (size_t)l->cout);
  for (int i = 0; i < x->n; ++i)
    for (int oy = 0; oy < oh; ++oy)
      for (int ox = 0; ox < ow; ++ox) {
        memset(si, 0, 4 * (size_t)l->cout);
        memset(sf, 0, 4 * (size_t)l->cout);
        for (int t = 0; t < taps; ++t) {
          const int iy = oy * l->sh - l->pt + t / l->kw, ix = ox * l->sw - l->pl + t % l->kw;
          const int64_t at = tpix(x, i, iy, ix); /* inside the border by construction */
          if (l->int8) {
            const uint8_t* a = x->b + at;
            if (dw) {
              for (int j = 0; j < l->cout; ++j) si[j] += ((int32_t)a[j] - xv->zero) * l->wt[(size_t)t * l->cout + j];
            } else {
              for (int c = 0; c < l->cin; ++c) {
                const int32_t av = (int32_t)a[c] - xv->zero;
                const int32_t* w = l->wt + ((size_t)t * cpg + c) * l->cout;
                for (int j = 0; j < l->cout; ++j) si[j] += av * w[j];
              }
            }
          } else {
            const float* a = x->f + at;
            if (dw) {
              for (int j = 0; j < l->cout; ++j) sf[j] = fmaf(a[j], l->wtf[(size_t)t * l->cout + j], sf[j]);
            } else {
              for (int c = 0; c < l->cin; ++c) {
                const float av = a[c];
                const float* w = l->wtf + ((size_t)t * cpg + c) * l->cout;
                for (int j = 0; j < l->cout; ++j) sf[j] = fmaf(av, w[j], sf[j]);
              }
            }
          }
        }
        const int64_t d = tpix(y, i, oy, ox);
        const int64_t ri = r ? tpix(r, i, oy / l->res_fh, ox >> l->res_shift) : 0;
        for (int j = 0; j < l->cout; ++j) {
          const float v = epi_float(l->int8 ? (float)si[j] : sf[j], l, j, r, rv, ri + j);
          if (u8)
            y->b[d + j] = requant(v, ov);
          else
            y->f[d + j] = v;
        }
      }
  free(si);
  free(sf);
}

/* The recognizer on n crops [n][height][bw] (uint8 page bytes): logits [n][classes][T] (the
 * reference's to_nchw: a uint8 output read through table[q] = (q - zero) * scale,
 * net.cpp:1101-1128).  keep_value >= 0: that value's NHWC bytes (uint8) or floats, without its
 * border, copied to keep_out (for layer-by-layer checks).  Returns T, or < 0 on an error. */
ORC_API int orc_model_run(void* h, const uint8_t* crops, int n, int bw, float* logits, int keep_value,
                          void* keep_out) {
  orc_model* m = (orc_model*)h;
  tens* vals = (tens*)calloc((size_t)m->nv, sizeof(tens));
  const orc_value* xv = &m->v[m->inp];
  tens_alloc(&vals[m->inp], xv, m->quantized && xv->u8, n, m->height, bw);
  uint8_t table[256];
  if (m->quantized) orc_input_table(m, table);
  for (int i = 0; i < n; ++i)
    for (int y = 0; y < m->height; ++y)
      for (int x = 0; x < bw; ++x) {
        const uint8_t p = crops[((size_t)i * m->height + y) * bw + x];
        const int64_t d = tpix(&vals[m->inp], i, y, x);
        if (m->quantized)
          vals[m->inp].b[d] = table[p];
        else
          vals[m->inp].f[d] = 1.0f - (float)p / 255.0f;
      }
  for (int k = 0; k < m->nl; ++k) run_layer(m, &m->l[k], vals);
  const tens* o = &vals[m->outv];
  const orc_value* ov = &m->v[m->outv];
  const int frames = o->h * o->w;
  float tab[256];
  for (int q = 0; q < 256; ++q) tab[q] = (float)(q - ov->zero) * ov->scale;
  if (logits)
    for (int i = 0; i < n; ++i)
      for (int y = 0; y < o->h; ++y)
        for (int x = 0; x < o->w; ++x) {
          const int64_t s = tpix(o, i, y, x);
          for (int c = 0; c < o->c; ++c)
            logits[((size_t)i * o->c + c) * frames + y * o->w + x] = o->b ? tab[o->b[s + c]] : o->f[s + c];
        }
  if (keep_value >= 0 && keep_value < m->nv && keep_out) {
    const tens* t = &vals[keep_value];
    size_t at = 0;
    for (int i = 0; i < t->n; ++i)
      for (int y = 0; y < t->h; ++y)
        for (int x = 0; x < t->w; ++x) {
          const int64_t s = tpix(t, i, y, x);
          if (t->b) {
            memcpy((uint8_t*)keep_out + at, t->b + s, (size_t)t->c);
          } else {
            memcpy((float*)keep_out + at, t->f + s, 4 * (size_t)t->c);
          }
          at += (size_t)t->c;
        }
  }
  for (int k = 0; k < m->nv; ++k) {
    free(vals[k].b);
    free(vals[k].f);
  }
  free(vals);
  return frames;
}

/* ------------------------------------------------------------------ CTC */

/* carbon/src/cpu/kernels.h:216-250 (exp_neg): x clamped to -87, n = round(x log2 e) half to even,
 * r = x - n ln2 in two parts (Cody and Waite), Cephes's degree-5 polynomial, times 2^n through
 * the exponent bits; every multiply and add on its own, in this order. */
ORC_API float orc_exp_neg(float x) {
  x = x > -87.0f ? x : -87.0f;
  const float n = nearbyintf(x * 1.44269504088896341f);
  float r = x - n * 0.693359375f;
  r = r - n * -2.12194440e-4f;
  float p = 1.9875691500e-4f;
  p = p * r + 1.3981999507e-3f;
  p = p * r + 8.3334519073e-3f;
  p = p * r + 4.1665795894e-2f;
  p = p * r + 1.6666665459e-1f;
  p = p * r + 5.0000001201e-1f;
  const float y = p * (r * r) + r + 1.0f;
  const int32_t bits = ((int32_t)n + 127) << 23;
  float s;
  memcpy(&s, &bits, 4);
  return y * s;
}

/* carbon/src/cpu/kernels.cpp:799-828 (ctc_argmax, the scalar reference): per frame t < t_n the
 * best class (ties to the lower id); for a non-blank best, 1 / sum over classes in order of
 * exp_neg(l_c - l_best). */
static void ctc_argmax(const float* logits, int classes, int frames, int t_n, int32_t* ids, float* probs) {
  for (int t = 0; t < t_n; ++t) {
    float best = -INFINITY;
    int32_t arg = 0;
    for (int c = 0; c < classes; ++c) {
      const float v = logits[(size_t)c * frames + t];
      if (v > best) {
        best = v;
        arg = c;
      }
    }
    ids[t] = arg;
    if (arg == 0) continue;
    float sum = 0.0f;
    for (int c = 0; c < classes; ++c) sum = sum + orc_exp_neg(logits[(size_t)c * frames + t] - best);
    probs[t] = 1.0f / sum;
  }
}

/* carbon/src/lines.cpp:331-355 (ctc_collapse) over per-frame ids and probs; then
 * carbon/src/lines.cpp:357-370 (ctc_greedy).  Per line: its count, and up to cap ids, first
 * frames and max probs at i * cap. */
ORC_API void orc_ctc_collapse(const int32_t* ids, const float* probs, int n, int frames, const int32_t* lengths,
                              int cap, int32_t* counts, int32_t* out_ids, int32_t* out_frames, float* out_probs) {
  for (int i = 0; i < n; ++i) {
    int t_n = lengths[i] < 0 ? 0 : lengths[i] > frames ? frames : lengths[i];
    const int32_t* a = ids + (size_t)i * frames;
    const float* q = probs ? probs + (size_t)i * frames : NULL;
    int k = 0, prev = 0;
    for (int t = 0; t < t_n; ++t) {
      const int id = a[t];
      const float p = q ? q[t] : 1.0f;
      if (id != 0 && id != prev) {
        if (k < cap) {
          out_ids[(size_t)i * cap + k] = id;
          out_frames[(size_t)i * cap + k] = t;
          out_probs[(size_t)i * cap + k] = p;
        }
        ++k;
      } else if (id != 0 && k - 1 < cap) {
        float* last = &out_probs[(size_t)i * cap + k - 1];
        *last = *last > p ? *last : p;
      }
      prev = id;
    }
    counts[i] = k;
  }
}

ORC_API void orc_ctc_greedy(const float* logits, int n, int classes, int frames, const int32_t* lengths, int cap,
                            int32_t* counts, int32_t* out_ids, int32_t* out_frames, float* out_probs,
                            int32_t* frame_ids, float* frame_probs) {
  int32_t* arg = (int32_t*)calloc((size_t)n * frames, 4);
  float* prob = (float*)calloc((size_t)n * frames, 4);
  for (int i = 0; i < n; ++i) {
    int t_n = lengths[i] < 0 ? 0 : lengths[i] > frames ? frames : lengths[i];
    ctc_argmax(logits + (size_t)i * classes * frames, classes, frames, t_n, arg + (size_t)i * frames,
               prob + (size_t)i * frames);
  }
  orc_ctc_collapse(arg, prob, n, frames, lengths, cap, counts, out_ids, out_frames, out_probs);
  if (frame_ids) memcpy(frame_ids, arg, 4 * (size_t)n * frames);
  if (frame_probs) memcpy(frame_probs, prob, 4 * (size_t)n * frames);
  free(arg);
  free(prob);
}

/* carbon/src/cpu/kernels.cpp:617-665 (ctc_topk, the scalar reference; carbon::frame_candidates,
 * carbon/src/beam.cpp:301-310): of one line's logits [classes][frames], its first t_n frames:
 * each frame's best logit, the class-order sum of exp_neg(l_c - best), its k likeliest classes
 * but the blank by insertion in class order (a later class must beat a kept one, so ties keep
 * the lower id), ids[t * k + j]; logp[t * k + j] and blank[t] each the logit less best + logf(sum)
 * (the C library's logf, as std::log(float) is). */
ORC_API void orc_ctc_topk(const float* logits, int classes, int frames, int t_n, int k, int32_t* ids, float* logp,
                          float* blank) {
  for (int t = 0; t < t_n; ++t) {
    float best = -INFINITY, sum = 0.0f;
    for (int c = 0; c < classes; ++c) {
      const float v = logits[(size_t)c * frames + t];
      best = v > best ? v : best;
    }
    for (int c = 0; c < classes; ++c) sum = sum + orc_exp_neg(logits[(size_t)c * frames + t] - best);
    float* lt = logp + (size_t)t * k;
    int32_t* it = ids + (size_t)t * k;
    for (int j = 0; j < k; ++j) {
      lt[j] = -INFINITY;
      it[j] = 0;
    }
    for (int c = 1; c < classes && k > 0; ++c) {
      const float v = logits[(size_t)c * frames + t];
      if (!(v > lt[k - 1])) continue;
      int j = k - 1;
      for (; j > 0 && lt[j - 1] < v; --j) {
        lt[j] = lt[j - 1];
        it[j] = it[j - 1];
      }
      lt[j] = v;
      it[j] = c;
    }
    const float off = best + logf(sum);
    for (int j = 0; j < k; ++j) lt[j] = lt[j] - off;
    blank[t] = logits[t] - off;
  }
}
