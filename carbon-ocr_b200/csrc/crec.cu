// The C ABI (include/carbon_rec.h) over the sm_100a kernels: the model blob read into device
// weights, the group layout, tensor maps, launches and results.
//
// A run's lines lie end to end along the width of one tensor per layer: line i at input
// columns [seg_i, seg_i + bw_i), gaps of `gap` columns between them (and before the first)
// holding the zero point, so every convolution of every line reads exactly the borders the
// reference's executor gives a batch of that bucket width (carbon/src/net/net.cpp:100-160),
// and each layer is one launch over the whole run whatever the mix of widths.  A gap is as
// wide as the widest padding any layer reads, in input columns; segments and gaps are whole
// multiples of the network's horizontal stride.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <condition_variable>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <type_traits>
#include <vector>

#include "../../include/carbon_rec.h"
#include "conv_gemm.cuh"
#include "crop_stem.cuh"
#include "ctc.cuh"
#include "dw_head.cuh"
#include "peak.cuh"
#include "sm100.cuh"
#include "host_pool.h"
#include "stager.h"

using namespace crec;

namespace {

constexpr int kKindConv = 0, kKindDw = 1, kKindResize = 2;
// Band mode (conv_gemm.cuh) is bit-exact but off: it gathers its channel planes 16 bytes at a time
// from NHWC rows, which from L2 was 1.6x faster than the im2col windows (s1b of a 524,288-column
// run, 46 against 76 us) but from DRAM, at full run size, 2x slower (s1b 5.1 against 2.6 ms a
// step).  It needs its input written chunk-planar by the layer before.
constexpr bool kNoBand = true;
constexpr size_t kGuard = 64 << 10;
constexpr int kPoolLines = 2048;    // a run's layout goes to the host pool from this many lines
constexpr int kOrderBuckets = 1024;  // the crop kernel's claim order: a counting sort's buckets
constexpr int kStagerWorkers = 8;    // at most, threads staging pageable page rows through pinned chunks

struct Value {
  int c = 0, u8 = 0, ph = 0, pw = 0, zero = 0;
  float scale = 1.0f;
  // layout
  int h = 0;       // rows
  int shift = 0;   // log2 of input columns per column
  int phys = -1;   // the value whose memory holds it (itself, or a Resize's source)
  int extra = 0;   // log2 of the nearest upsampling read in place: physical column = column >> extra
  int cp = 0;      // channels padded to 16
  bool real = false;
  uint8_t* alloc = nullptr;
  uint8_t* base = nullptr;  // first (top border) row
  long long pitch = 0;      // bytes a row
  size_t bytes = 0;
};

struct Layer {
  int kind, in, out, residual, kh, kw, sh, sw, pt, pl, pb, pr, cin, cout, relu, fh, fw, res_fh, res_shift, int8;
  std::vector<int8_t> w8;  // [cout][cin/g][kh][kw]
  std::vector<float> wf, wsc, bias;
  // device
  uint8_t* wimg = nullptr;
  int32_t* colsum = nullptr;
  float* scale = nullptr;
  float* dbias = nullptr;
  int8_t* dw8 = nullptr;  // depthwise [taps][cp], stem [cout][taps], head [cout][input cp]
  float* dwf = nullptr;
  int32_t* hoff = nullptr;  // the INT8 epilogue's per-channel offsets (HeadParams::off, ConvParams::off, DwParams::off)
  uint32_t* dwt = nullptr;  // the INT8 row depthwise's tap-transposed weights (DwParams::wt)
  uint32_t* dwc = nullptr;  // and its per-channel constants (DwParams::dwc)
  bool fast = false;        // its sums fit the exact conversions without the conversion unit
  bool sat = false;         // INT8 conv: |v * inv_scale| < 2^21 always (round, then clamp while packing)
  int nkb = 0, last_steps = 0, nt = 0, n_tiles = 0, stages = 0, nchunk = 0, chunks = 0;
  int krows = 0, q_rows = 1, cq = 0;  // dense convs: input rows a tile reads, output rows it stacks, channels a row
  // row stacking (ConvParams::st_*): the output rows input row i serves, its weight block's offset
  int st_q0[kMaxKRows] = {}, st_n[kMaxKRows] = {};
  uint32_t st_off[kMaxKRows] = {}, st_first = 0;
  int tail = 128;           // the last K block's row bytes (ConvParams::tail_bytes)
  uint32_t row_bytes = 0;   // without row stacking: an input row's weight blocks (ConvParams::row_bytes)
  uint32_t stage_bytes = 0, a_bytes = 0, b_bytes = 0, smem = 0;
  // band mode (conv_gemm.cuh): channel-plane ring slots, resident weights
  bool band = false;
  int pairs = 0, band_chunks = 0, plane_px = 0, band_rows = 0, gx0 = 0;
  int kx_parity[3] = {0, 0, 0}, kx_off[3] = {0, 0, 0};
  uint32_t slot_bytes = 0, load_bytes = 0, w_bytes = 0;
};

template <class T>
T rd(const uint8_t*& p) {
  T v;
  std::memcpy(&v, p, sizeof v);
  p += sizeof v;
  return v;
}

long long round_up(long long v, long long m) { return (v + m - 1) / m * m; }
int round16(int v) { return (v + 15) / 16 * 16; }
int log2i(int v) {
  int s = 0;
  while ((1 << s) < v) ++s;
  return (1 << s) == v ? s : -1;
}

// carbon/src/net/net.cpp:84-90 (quantize), the input table's arithmetic.
uint8_t quantize_in(float v, float scale, int zero) {
  float r = v / scale;
  r = std::min(4194304.0f, std::max(-4194304.0f, r));
  volatile float t = r + 12582912.0f;
  r = t - 12582912.0f;
  r += static_cast<float>(zero);
  return static_cast<uint8_t>(std::min(255.0f, std::max(0.0f, r)));
}

uint16_t half_bits(float f) {
  const __half h = __float2half_rn(f);
  uint16_t b;
  std::memcpy(&b, &h, 2);
  return b;
}
float half_round(float f) { return __half2float(__float2half_rn(f)); }

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

}  // namespace

struct crec_handle {
  crec_config cfg{};
  std::string error;
  bool broken = false;
  int device = 0, sms = 0;
  bool int8 = true;
  int eb = 1;
  cudaStream_t stream = nullptr;
  EncodeTiled encode = nullptr;
  // model
  std::vector<Value> v;
  std::vector<Layer> l;
  int inp = 0, outv = 0, height = 32;
  int gap = 8, max_shift = 0, head_shift = 0;
  long long max_cols = 0;  // input columns a run holds
  uint8_t* in_table = nullptr;
  float* head_table = nullptr;
  float* ctc_terms = nullptr;  // INT8: [256][256] exp_neg(table[q] - table[best])
  // INT8: a run's non-blank frames for the class-order sums (the head lists them, ctc_sums_kernel adds)
  uint8_t* d_nb_codes = nullptr;  // [frames][nb_row_bytes]
  int32_t* d_nb_frame = nullptr;
  int32_t* d_nb_best = nullptr;
  int* d_nb_count = nullptr;  // [CTA][2]: listed, 255 - least best code
  int nb_row_bytes = 0;
  // pages: two slots, the group being read and the next group's upload (prefetch_pages, on the
  // copy stream while the current group's runs go on), as the reference's CUDA device keeps them
  // (carbon/src/cuda/pipeline_cuda.cpp:407-437); or the caller's own device pages
  struct PageSlot {
    uint8_t* mem = nullptr;
    size_t cap = 0;
    PageDesc* d_pages = nullptr;     // [max_pages]
    std::vector<PageDesc> pages;     // device pointers
    std::vector<crec_page> views;    // the host pages uploaded (what set_pages compares)
    cudaEvent_t done = nullptr;      // its upload, recorded on the copy stream
    cudaEvent_t unused = nullptr;    // the last recognize work that read it, on the recognize stream
    bool ready = false;              // a prefetch's upload set_pages has not taken yet
    bool recorded = false;           // `unused` recorded
    long long bytes = 0;             // what its last upload sent
  };
  PageSlot slot[2];
  int cur = 0;
  cudaEvent_t last_upload = nullptr;  // the previous set_pages / prefetch_pages call's upload
  cudaStream_t copy_stream = nullptr;
  // pageable pages go through the stager's pinned chunks (made on first use); prefetch_pages hands
  // its upload to the uploader thread and returns, as the reference's CudaModels does
  // (carbon/src/cuda/pipeline_cuda.cpp:422-437, 654-672)
  std::unique_ptr<crec::Stager> stager;
  std::thread up_thread;
  std::mutex up_m;
  std::condition_variable up_cv;
  bool up_stop = false, up_busy = false;
  struct UpJob {
    PageSlot* slot = nullptr;
    std::vector<crec_page> pages;
    std::vector<std::vector<int32_t>> runs;  // copies of the caller's row runs
    bool has_rows = false;
  } up_job;
  PageDesc* d_ext_pages = nullptr;  // set_pages_device's descriptors
  std::vector<PageDesc> pages;      // the current group's, device pointers
  PageDesc* d_pages = nullptr;      // and their descriptors on the device
  int max_pages = 0;
  // run buffers
  LineDesc* d_lines = nullptr;
  int* d_claim = nullptr;  // the crop kernel's line claims: [2], 0 between launches
  int* d_order = nullptr;  // [max_lines] a run's lines in claim order
  int* hs_order = nullptr;  // a call's claim orders, each run's from its first line's index (pinned)
  size_t cap_hs_order = 0;
  std::vector<int> order_count;  // the counting sort's buckets
  std::vector<int> hs_key;       // a call's lines' claim keys
  std::unique_ptr<crec::HostPool> pool;  // the layout's threads (made for the first large run)
  // lines beyond the crop kernel's reach: a run's list (slot order) on the device, their raw crops
  // (grown on demand), and the run's widest filter and tallest source span among them
  int* d_wide_idx = nullptr;
  uint8_t* d_wide = nullptr;
  size_t cap_wide = 0;
  int* hs_wide = nullptr;  // a call's lists, each run's from its first line's index (pinned)
  size_t cap_hs_wide = 0;
  int run_wide = 0, run_vtaps = 0, run_htaps = 0, run_rows = 0;
  long long st_wide = 0;  // the last call's wide lines
  uint8_t* d_mask = nullptr;
  int* d_frame0 = nullptr;
  int* d_length = nullptr;
  // a call's pinned staging (grown on demand): line descriptors, masks, frame starts, lengths, results
  LineDesc* hs_lines = nullptr;
  int* hs_frame0 = nullptr;
  int* hs_length = nullptr;
  uint8_t* hs_mask = nullptr;
  size_t cap_lines = 0, cap_frame0 = 0, cap_length = 0, cap_mask = 0;
  // a call's packed decodings on the device (grown on demand): every line's count and offset, the
  // characters end to end, the running total
  int32_t* dp_counts = nullptr;
  int32_t* dp_offsets = nullptr;
  int32_t* dp_ids = nullptr;
  int32_t* dp_frames = nullptr;
  float* dp_probs = nullptr;
  long long* d_total = nullptr;
  long long* h_total = nullptr;  // pinned
  // a call's running total after each run but the last (pinned), recorded with the run's event, so
  // the run's decodings are read back while the next run computes (on the readback stream)
  long long* h_run_total = nullptr;
  size_t cap_run_total = 0;
  std::vector<cudaEvent_t> ev_run;
  cudaStream_t read_stream = nullptr;
  size_t cap_dp_lines = 0, cap_dp_chars = 0;
  int32_t* d_frame_id = nullptr;
  float* d_frame_prob = nullptr;
  int32_t* d_count = nullptr;
  int32_t* d_ids = nullptr;
  int32_t* d_frames = nullptr;
  float* d_probs = nullptr;
  int* d_err = nullptr;
  int* h_err = nullptr;
  uint8_t* d_crops = nullptr;  // debug copy of the finished crops
  int crops_pitch = 0;
  float* d_logits = nullptr;  // test hook: the last run's logits, [columns at the head's resolution][classes]
  uint8_t* d_crops_in = nullptr;  // ready crops given by crec_recognize_crops
  int crops_in_pitch = 0;
  const uint8_t* run_crops = nullptr;  // this run's ready crops on the device, or null
  const int* run_bw = nullptr;         // this run's bucket widths (host)
  // the last call's statistics, and the optional per-launch profile (CUDA events on the stream)
  long long st_runs = 0, st_launches = 0, st_h2d = 0, st_d2h = 0;
  long long tot_h2d = 0, tot_d2h = 0;  // since open, the calls' own
  long long up_h2d = 0;                // since open, the uploader's (under up_m)
  bool profile = false;
  std::vector<cudaEvent_t> ev_pool;  // pairs
  std::vector<int> ev_kind;          // a pair's kernel kind
  std::vector<int> ev_layer;         // and its layer (the layer count for the collapse)
  size_t ev_used = 0;
  double prof_ms[8] = {0}, prof_ops[8] = {0};
  long long prof_count[8] = {0};
  std::vector<double> lprof_ms, lprof_ops;  // by layer (and the collapse after the last)
  std::vector<long long> lprof_count;
  // test hooks (crec_debug_inject), armed for the next run
  bool inject_timeout = false, inject_sticky = false;
  // the last run
  int last_n = 0;
  int last_a = 0;                          // the last run's first line in its call
  std::vector<int> last_frame0, last_len;  // its lines' first frame columns and lengths (the beam's candidates)
  // crec_candidates' buffers (grown on demand)
  int32_t* d_cand_cols = nullptr;
  int32_t* d_cand_ids = nullptr;
  float* d_cand_vals = nullptr;
  float* d_cand_fr = nullptr;  // [3][frames]: best, sum, the blank's logit
  size_t cap_cand_frames = 0, cap_cand_cells = 0;
  long long last_cols = 0;
  std::vector<int> last_seg, last_bw;
};

namespace {

int set_error(crec_handle* h, int code, const std::string& msg) {
  if (h) h->error = msg;
  return code;
}

int cuda_status(crec_handle* h, cudaError_t e, const char* what) {
  if (e == cudaSuccess) return CREC_OK;
  // the errors after which a context can run nothing more (carbon/src/cuda/pipeline_cuda.cpp:344-363)
  switch (e) {
    case cudaErrorIllegalAddress:
    case cudaErrorLaunchFailure:
    case cudaErrorIllegalInstruction:
    case cudaErrorMisalignedAddress:
    case cudaErrorInvalidAddressSpace:
    case cudaErrorInvalidPc:
    case cudaErrorHardwareStackError:
    case cudaErrorAssert:
    case cudaErrorECCUncorrectable:
    case cudaErrorDevicesUnavailable:
    case cudaErrorLaunchTimeout:
    case cudaErrorUnknown:
      h->broken = true;
      return set_error(h, CREC_E_STICKY, std::string(what) + ": " + cudaGetErrorString(e));
    case cudaErrorMemoryAllocation:
      cudaGetLastError();
      return set_error(h, CREC_E_NOMEM, std::string(what) + ": " + cudaGetErrorString(e));
    default:
      cudaGetLastError();
      return set_error(h, CREC_E_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  }
}

#define CK(call)                                           \
  do {                                                     \
    const int rc_ = cuda_status(h, (call), #call);         \
    if (rc_ != CREC_OK) return rc_;                        \
  } while (0)

template <class T>
int dev_alloc(crec_handle* h, T** p, size_t count) {
  CK(cudaMalloc(reinterpret_cast<void**>(p), std::max<size_t>(count, 1) * sizeof(T)));
  return CREC_OK;
}
template <class T>
int host_alloc(crec_handle* h, T** p, size_t count) {
  CK(cudaHostAlloc(reinterpret_cast<void**>(p), std::max<size_t>(count, 1) * sizeof(T), cudaHostAllocDefault));
  return CREC_OK;
}
template <class T>
int upload(crec_handle* h, T** d, const std::vector<T>& v) {
  int rc = dev_alloc(h, d, v.size());
  if (rc) return rc;
  if (!v.empty()) CK(cudaMemcpy(*d, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice));
  return CREC_OK;
}

// The model blob (carbon_rec/netdef.py, RecNet.to_blob).
int read_model(crec_handle* h, const uint8_t* blob, size_t len) {
  if (!blob || len < 48 || std::memcmp(blob, "CRECMDL1", 8) != 0) return set_error(h, CREC_E_MODEL, "not a CRECMDL1 model blob");
  const uint8_t* p = blob + 8;
  const uint8_t* end = blob + len;
  if (rd<uint32_t>(p) != 1) return set_error(h, CREC_E_MODEL, "model blob version");
  const uint32_t kind = rd<uint32_t>(p);
  const uint32_t nv = rd<uint32_t>(p), nl = rd<uint32_t>(p);
  h->inp = static_cast<int>(rd<uint32_t>(p));
  h->outv = static_cast<int>(rd<uint32_t>(p));
  h->height = static_cast<int>(rd<uint32_t>(p));
  rd<uint32_t>(p);
  if ((kind == 0) != h->int8)
    return set_error(h, CREC_E_MODEL, h->int8 ? "CREC_INT8 needs the Q/DQ file's blob" : "CREC_FP16 needs the float file's blob");
  if (nv > 4096 || nl > 4096) return set_error(h, CREC_E_MODEL, "model blob sizes");
  h->v.resize(nv);
  for (auto& v : h->v) {
    if (p + 24 > end) return set_error(h, CREC_E_MODEL, "model blob truncated");
    v.c = static_cast<int>(rd<uint32_t>(p));
    v.u8 = static_cast<int>(rd<uint32_t>(p));
    v.scale = rd<float>(p);
    v.zero = rd<int32_t>(p);
    v.ph = static_cast<int>(rd<uint32_t>(p));
    v.pw = static_cast<int>(rd<uint32_t>(p));
    if (!h->int8) {
      v.u8 = 0;
      v.zero = 0;
    }
  }
  h->l.resize(nl);
  for (auto& l : h->l) {
    if (p + 84 > end) return set_error(h, CREC_E_MODEL, "model blob truncated");
    int* f = &l.kind;
    for (int k = 0; k < 20; ++k) f[k] = (k == 3) ? rd<int32_t>(p) : static_cast<int>(rd<uint32_t>(p));
    if (l.in < 0 || l.in >= static_cast<int>(nv) || l.out < 0 || l.out >= static_cast<int>(nv) ||
        l.residual >= static_cast<int>(nv))
      return set_error(h, CREC_E_MODEL, "model blob value index");
    if (l.kind == kKindResize) continue;
    const int groups = l.kind == kKindDw ? l.cin : 1;
    const size_t nw = static_cast<size_t>(l.cout) * (l.cin / groups) * l.kh * l.kw;
    if (l.int8) {
      if (p + ((nw + 3) / 4 * 4) + 4 * l.cout > end) return set_error(h, CREC_E_MODEL, "model blob truncated");
      l.w8.assign(reinterpret_cast<const int8_t*>(p), reinterpret_cast<const int8_t*>(p) + nw);
      p += (nw + 3) / 4 * 4;
      l.wsc.resize(l.cout);
      std::memcpy(l.wsc.data(), p, 4 * l.cout);
      p += 4 * l.cout;
    } else {
      if (p + 4 * nw > end) return set_error(h, CREC_E_MODEL, "model blob truncated");
      l.wf.resize(nw);
      std::memcpy(l.wf.data(), p, 4 * nw);
      p += 4 * nw;
    }
    if (p + 4 * l.cout > end) return set_error(h, CREC_E_MODEL, "model blob truncated");
    l.bias.resize(l.cout);
    std::memcpy(l.bias.data(), p, 4 * l.cout);
    p += 4 * l.cout;
  }
  if (p != end) return set_error(h, CREC_E_MODEL, "model blob has trailing bytes");
  return CREC_OK;
}

// Shapes through the network, which values need memory, the gap; refuses what the kernels do not run.
int plan_model(crec_handle* h) {
  auto& V = h->v;
  auto& L = h->l;
  if (L.size() < 2) return set_error(h, CREC_E_MODEL, "a recognizer of at least a stem and a head");
  for (auto& v : V) v.h = -1;
  V[h->inp].h = h->height;
  V[h->inp].shift = 0;
  V[h->inp].phys = h->inp;
  for (size_t i = 0; i < L.size(); ++i) {
    const Layer& l = L[i];
    Value& x = V[l.in];
    Value& y = V[l.out];
    if (x.h < 0) return set_error(h, CREC_E_MODEL, "layers out of order");
    if (l.kind == kKindResize) {
      const int s = log2i(l.fw);
      if (l.fh != 1 || s < 0 || s > x.shift) return set_error(h, CREC_E_MODEL, "a Resize other than a 2^k widening");
      y.h = x.h;
      y.shift = x.shift - s;
      y.phys = x.phys;
      y.extra = x.extra + s;
      continue;
    }
    const int s = log2i(l.sw);
    if (s < 0 || l.kh > 3 || l.res_fh != 1) return set_error(h, CREC_E_MODEL, "a convolution this build does not run");
    y.h = (x.h + l.pt + l.pb - l.kh) / l.sh + 1;
    y.shift = x.shift + s;
    y.phys = l.out;
    y.extra = 0;
    y.real = true;
    if (i == 0) {
      if (l.in != h->inp || l.kind != kKindConv || l.cin != 1 || l.kh * l.kw > 9 || l.residual >= 0 || l.cout > kStemMaxOut ||
          l.pt != l.pb || l.pl != l.pr)
        return set_error(h, CREC_E_MODEL, "the first layer must be a 1-channel convolution of at most 3x3");
    } else if (static_cast<int>(i) == static_cast<int>(L.size()) - 1) {
      if (l.out != h->outv || l.kind != kKindConv || l.kh != 1 || l.kw != 1 || y.h != 1 || l.residual >= 0)
        return set_error(h, CREC_E_MODEL, "the last layer must be a 1x1 head on one row");
      if (h->int8 && !y.u8) return set_error(h, CREC_E_MODEL, "the INT8 head's output must be quantized (Q/DQ)");
      if (x.extra) return set_error(h, CREC_E_MODEL, "a head reading an upsampling");
      y.real = false;  // fused with CTC: never written
    } else {
      if (l.in == h->inp) return set_error(h, CREC_E_MODEL, "only the first layer reads the input");
      if (l.kind == kKindConv && x.extra) return set_error(h, CREC_E_MODEL, "a dense convolution reading an upsampling");
      if (l.kind == kKindDw && (l.sh != 1 || l.sw != 1)) return set_error(h, CREC_E_MODEL, "a strided depthwise convolution");
    }
    if (l.int8 != (h->int8 ? 1 : 0)) return set_error(h, CREC_E_MODEL, "mixed int8 and float layers");
  }
  int max_shift = 0, gap = 1;
  for (auto& v : V) {
    if (v.h < 0) continue;
    max_shift = std::max(max_shift, v.shift + v.extra);
    gap = std::max(gap, v.pw << v.shift);
    v.cp = round16(std::max(v.c, 1));
  }
  h->max_shift = max_shift;
  h->gap = static_cast<int>(round_up(gap, std::max(8, 1 << max_shift)));
  h->head_shift = V[h->outv].shift;
  return CREC_OK;
}

// The 128-byte swizzle of a K-major operand block: byte b of row j.
inline size_t swz(int j, int b) { return static_cast<size_t>(j) * 128 + (((b >> 4) ^ (j & 7)) << 4) + (b & 15); }
// Byte b of row j of a K-major block whose rows are `pitch` bytes (128, 64 or 32) in that width's
// swizzle: the 16-byte chunk index XOR the row's bits above the atom's (Swizzle<3|2|1, 4, 3>).
inline size_t swz_pitch(int j, int b, int pitch) {
  const int chunks = pitch / 16, mask = chunks - 1;
  const int shift = pitch == 128 ? 0 : pitch == 64 ? 1 : 2;
  return static_cast<size_t>(j) * pitch + ((((b >> 4) ^ (j >> shift)) & mask) << 4) + (b & 15);
}

// A dense layer's (or the head's) weights as the swizzled image the kernels bulk-copy:
// [n tile][ky][kb][nt rows][128 bytes]; byte `off` of kernel row ky's window is (kx, channel, byte).
std::vector<uint8_t> weight_image(const crec_handle* h, const Layer& l, int cp_in, int nt, int n_tiles, int nkb) {
  const int eb = h->eb, taps = l.kh * l.kw, window = l.kw * cp_in * eb;
  // blocks [n tile][input row i][kb]; tile column j is output row q = j / cq of the tile's
  // stacked rows, channel co; it reads input row i through kernel row i - q * sh (zeros where
  // that is outside the kernel).  A block has nt rows of 128 bytes, the last kb's of l.tail.
  const size_t row_bytes = static_cast<size_t>(nkb - 1) * nt * 128 + static_cast<size_t>(nt) * l.tail;
  std::vector<uint8_t> img(static_cast<size_t>(n_tiles) * l.krows * row_bytes, 0);
  for (int n = 0; n < n_tiles; ++n)
    for (int i = 0; i < l.krows; ++i)
      for (int kb = 0; kb < nkb; ++kb) {
        uint8_t* blk = img.data() + static_cast<size_t>(n * l.krows + i) * row_bytes + static_cast<size_t>(kb) * nt * 128;
        const int pitch = kb == nkb - 1 ? l.tail : 128;
        for (int j = 0; j < nt; ++j) {
          const int q = l.q_rows > 1 ? j / l.cq : 0;
          const int co = n * nt + j - q * l.cq, ky = i - q * l.sh;
          if (co >= l.cout || ky < 0 || ky >= l.kh) continue;
          for (int b = 0; b < pitch; ++b) {
            const int off = kb * 128 + b;
            if (off >= window) break;
            const int kx = off / (cp_in * eb), rem = off % (cp_in * eb), c = rem / eb, byte = rem % eb;
            if (c >= l.cin) continue;
            const size_t wi = (static_cast<size_t>(co) * l.cin + c) * taps + ky * l.kw + kx;
            uint8_t val;
            if (h->int8) {
              val = static_cast<uint8_t>(l.w8[wi]);
            } else {
              const uint16_t hb = half_bits(l.wf[wi]);
              val = static_cast<uint8_t>(byte ? hb >> 8 : hb & 0xff);
            }
            blk[swz_pitch(j, b, pitch)] = val;
          }
        }
      }
  return img;
}

// A dense layer's weights in band mode: [ky][kx][32-byte channel pair][nt / 8][2 chunks][8 rows][16
// bytes], the tensor cores' K-major layout without swizzle (zeros past the input's channels and
// past cout).
std::vector<uint8_t> band_weight_image(const crec_handle* h, const Layer& l, int nt) {
  const int eb = h->eb, taps = l.kh * l.kw;
  std::vector<uint8_t> img(static_cast<size_t>(taps) * l.pairs * nt * 32, 0);
  for (int ky = 0; ky < l.kh; ++ky)
    for (int kx = 0; kx < l.kw; ++kx)
      for (int pr = 0; pr < l.pairs; ++pr) {
        uint8_t* blk = img.data() + static_cast<size_t>((ky * l.kw + kx) * l.pairs + pr) * nt * 32;
        for (int n = 0; n < nt && n < l.cout; ++n)
          for (int c = 0; c < 2; ++c)
            for (int b = 0; b < 16; ++b) {
              const int byte = ((2 * pr + c) * 16 + b), ch = byte / eb;
              if (ch >= l.cin) continue;
              const size_t wi = (static_cast<size_t>(n) * l.cin + ch) * taps + ky * l.kw + kx;
              uint8_t v;
              if (h->int8) {
                v = static_cast<uint8_t>(l.w8[wi]);
              } else {
                const uint16_t hb = half_bits(l.wf[wi]);
                v = static_cast<uint8_t>(byte % 2 ? hb >> 8 : hb & 0xff);
              }
              blk[(n / 8) * 256 + c * 128 + (n % 8) * 16 + b] = v;
            }
      }
  return img;
}

// The INT8 epilogue's per-channel offsets (n of them) and whether its conversions may skip the
// conversion unit: a channel's sum(k) (a_k - zero) w_k over inputs a_k in [0, 255] lies in
// [-(zero P + (255 - zero) N), (255 - zero) P + zero N], P and N the sums of its positive weights
// and of its negative weights' magnitudes (both ends reached); below 2^22 in magnitude for every
// channel, the kernel converts exactly with kMagic.
int upload_offsets(crec_handle* h, Layer& l, int zero, const std::vector<int32_t>& colsum, int n) {
  const size_t per = l.w8.size() / static_cast<size_t>(l.cout);
  long long worst = 0;
  for (int j = 0; j < l.cout; ++j) {
    long long pos = 0, neg = 0;
    for (size_t k = 0; k < per; ++k) {
      const int w = l.w8[j * per + k];
      (w > 0 ? pos : neg) += std::abs(w);
    }
    worst = std::max({worst, (255 - zero) * pos + zero * neg, zero * pos + (255 - zero) * neg});
  }
  l.fast = worst < (1LL << 22);
  std::vector<int32_t> off(n, 0);
  for (int j = 0; j < n; ++j) {
    const int32_t zc = zero * colsum[j];
    off[j] = l.fast ? kMagicBits - zc : zc;
  }
  return upload(h, &l.hoff, off);
}

// Whether an INT8 layer's output stage may round before it clamps: the value before the clamp,
// v * inv_scale, bounded from the weights (|v| <= sum |w| * reach * scale + |bias| + 255 *
// residual scale, with a margin for the roundings) below 2^21, where the magic rounding is exact
// and clamping after rounding gives the same code (the bounds are integers).
bool round_first(const crec_handle* h, const Layer& l, const Value& x, const Value& y, const std::vector<float>& scale,
                 const std::vector<float>& bias) {
  const double reach = std::max(x.zero, 255 - x.zero);
  const double rs = l.residual >= 0 ? 255.0 * std::fabs(h->v[l.residual].scale) : 0.0;
  const size_t per = l.w8.size() / static_cast<size_t>(l.cout);
  double worst = 0.0;
  for (int j = 0; j < l.cout; ++j) {
    double a = 0.0;
    for (size_t k = 0; k < per; ++k) a += std::abs(static_cast<int>(l.w8[j * per + k]));
    worst = std::max(worst, a * reach * std::fabs(scale[j]) + std::fabs(bias[j]) + rs);
  }
  // a ReLU above a zero point clamps at the zero point, not at 0: left to the float clamp
  return worst * 1.01 * std::fabs(1.0 / y.scale) < static_cast<double>(1 << 21) && !(l.relu && y.zero > 0);
}

int setup_layer(crec_handle* h, size_t li) {
  Layer& l = h->l[li];
  if (l.kind == kKindResize) return CREC_OK;
  const Value& x = h->v[l.in];
  const Value& y = h->v[l.out];
  const int taps = l.kh * l.kw;
  const int cpo = li + 1 == h->l.size() ? 0 : y.cp;
  int rc;
  // per-channel constants, padded
  const int npad = std::max({cpo, round16(l.cout), 16}) + 256;
  std::vector<float> scale(npad, 0.0f), bias(npad, 0.0f);
  std::vector<int32_t> colsum(npad, 0);
  for (int j = 0; j < l.cout; ++j) {
    bias[j] = l.bias[j];
    if (h->int8) {
      scale[j] = x.scale * l.wsc[j];  // carbon/src/net/net.cpp:703
      const int per = l.kind == kKindDw ? 1 : l.cin;
      int32_t s = 0;
      for (int k = 0; k < per * taps; ++k) s += l.w8[static_cast<size_t>(j) * per * taps + k];
      colsum[j] = s;
    }
  }
  if ((rc = upload(h, &l.scale, scale)) || (rc = upload(h, &l.dbias, bias)) || (rc = upload(h, &l.colsum, colsum)))
    return rc;
  if (li == 0) {  // the stem: [cout][taps]
    if (h->int8) {
      l.sat = round_first(h, l, x, y, scale, bias);  // the stem's sums always fit the magic conversions
      if ((rc = upload(h, &l.dw8, l.w8))) return rc;
    } else {
      std::vector<float> wf(l.wf.size());
      for (size_t i = 0; i < wf.size(); ++i) wf[i] = half_round(l.wf[i]);
      if ((rc = upload(h, &l.dwf, wf))) return rc;
    }
    return CREC_OK;
  }
  if (l.kind == kKindDw) {  // [taps][cp]
    const int cp = y.cp;
    if (h->int8) l.sat = round_first(h, l, x, y, scale, bias);
    if (h->int8) {
      std::vector<int8_t> w(static_cast<size_t>(taps) * cp, 0);
      for (int c = 0; c < l.cout; ++c)
        for (int t = 0; t < taps; ++t) w[static_cast<size_t>(t) * cp + c] = l.w8[static_cast<size_t>(c) * taps + t];
      if ((rc = upload(h, &l.dw8, w))) return rc;
      if (l.kh == 1 && l.kw <= 12 && x.cp == cp) {  // the row kernel: channel c's taps 4j .. 4j+3 in slot j
        std::vector<uint32_t> wt(3 * static_cast<size_t>(cp), 0u), dc(3 * static_cast<size_t>(cp), 0u);
        for (int c = 0; c < cp; ++c) {
          for (int t = 0; t < l.kw && c < l.cout; ++t)
            wt[dw_row_index(t / 4, c, cp)] |= static_cast<uint32_t>(static_cast<uint8_t>(l.w8[static_cast<size_t>(c) * taps + t])) << (8 * (t % 4));
          const int32_t off = kMagicBits - x.zero * colsum[c];
          std::memcpy(&dc[dw_row_index(0, c, cp)], &off, 4);
          std::memcpy(&dc[dw_row_index(1, c, cp)], &scale[c], 4);
          std::memcpy(&dc[dw_row_index(2, c, cp)], &bias[c], 4);
        }
        if ((rc = upload(h, &l.dwt, wt)) || (rc = upload(h, &l.dwc, dc))) return rc;
      }
    } else {
      std::vector<float> w(static_cast<size_t>(taps) * cp, 0.0f);
      for (int c = 0; c < l.cout; ++c)
        for (int t = 0; t < taps; ++t) w[static_cast<size_t>(t) * cp + c] = half_round(l.wf[static_cast<size_t>(c) * taps + t]);
      if ((rc = upload(h, &l.dwf, w))) return rc;
    }
    return CREC_OK;
  }
  const int window = l.kw * x.cp * h->eb;
  l.nkb = (window + 127) / 128;
  l.last_steps = (window - (l.nkb - 1) * 128 + 31) / 32;
  if (li + 1 == h->l.size()) {  // the head
    if (l.nkb > 8) return set_error(h, CREC_E_MODEL, "a head reading more than 1024 bytes a frame");
    l.krows = 1;
    // a tile's frames stay resident (A: all K blocks) beside two class chunks of weights (B):
    // the widest chunk (N, up to 128 classes) with which that fits
    const uint32_t codes = h->int8 ? 128u * head_code_stride(l.cout) : 0u;
    l.a_bytes = static_cast<uint32_t>(l.nkb) * 16384;
    for (l.nchunk = std::min(kHeadChunk, round16(l.cout));; l.nchunk -= 16) {
      l.chunks = (l.cout + l.nchunk - 1) / l.nchunk;
      l.b_bytes = static_cast<uint32_t>(l.nkb) * l.nchunk * 128;
      l.smem = 1024 + l.a_bytes + 2 * l.b_bytes + codes + head_tail_bytes(l.chunks * l.nchunk, h->int8);
      if (l.smem + 1024 <= 232448) break;
      if (l.nchunk == 16) return set_error(h, CREC_E_MODEL, "the head does not fit in shared memory");
    }
    l.nt = l.nchunk;
    l.cq = l.nt;
    l.n_tiles = l.chunks;
    const int ncls = l.chunks * l.nchunk;
    // the weights [classes][x.cp], zeros past the real channels (the beam's candidates)
    if (h->int8) {
      std::vector<int8_t> w(static_cast<size_t>(l.cout) * x.cp, 0);
      for (int c = 0; c < l.cout; ++c)
        for (int j = 0; j < l.cin; ++j) w[static_cast<size_t>(c) * x.cp + j] = l.w8[static_cast<size_t>(c) * l.cin + j];
      if ((rc = upload(h, &l.dw8, w))) return rc;
    } else {
      std::vector<float> w(static_cast<size_t>(l.cout) * x.cp, 0.0f);
      for (int c = 0; c < l.cout; ++c)
        for (int j = 0; j < l.cin; ++j) w[static_cast<size_t>(c) * x.cp + j] = half_round(l.wf[static_cast<size_t>(c) * l.cin + j]);
      if ((rc = upload(h, &l.dwf, w))) return rc;
    }
    if (h->int8 && (rc = upload_offsets(h, l, x.zero, colsum, ncls))) return rc;
    if (h->int8) l.sat = round_first(h, l, x, y, scale, bias);
  } else {
    // row stacking: the number of output rows a tile computes that gets the most outputs from
    // an MMA (N up to 256; the rows divide the output's height; no residual), where that is at
    // least a quarter more than one row gets (measured: 1.2x predicted was no faster)
    const int cq = round16(l.cout), steps_row = (l.nkb - 1) * 4 + l.last_steps;
    double best = 0.0;
    l.q_rows = 1;
    for (int q = 1; q <= y.h && q * cq <= 256 && (q == 1 || l.residual < 0); ++q) {
      const int rows = (q - 1) * l.sh + l.kh;
      if (y.h % q || rows > kMaxKRows) continue;
      const double per_mma = static_cast<double>(q) / (rows * steps_row);
      if (per_mma > best * 1.001) {
        best = per_mma;
        l.q_rows = q;
      }
    }
    if (best < 1.25 / (l.kh * steps_row)) l.q_rows = 1;
    l.krows = (l.q_rows - 1) * l.sh + l.kh;
    l.nt = l.q_rows > 1 ? l.q_rows * cq : std::min(256, cq);
    l.cq = l.q_rows > 1 ? cq : l.nt;
    l.n_tiles = (y.cp + l.nt - 1) / l.nt;
    if (l.q_rows > 1) l.n_tiles = 1;
    l.a_bytes = 16384;
    l.b_bytes = static_cast<uint32_t>(l.nt) * 128;
    // a window's last K block of one or two 32-byte steps: boxes and weight rows that wide
    l.tail = l.last_steps <= 2 ? 32 * l.last_steps : 128;
    l.row_bytes = static_cast<uint32_t>(l.nkb - 1) * l.b_bytes + static_cast<uint32_t>(l.nt * l.tail);
    if (l.q_rows > 1) {
      // row stacking: input row i serves output rows q with 0 <= i - q * sh < kh, so its stages
      // carry those rows' weights only; a stage holds the most any input row needs
      int most = 0;
      l.st_first = 0;
      for (int i = 0; i < l.krows; ++i) {
        const int q0 = i < l.kh ? 0 : (i - l.kh + l.sh) / l.sh, q1 = std::min(l.q_rows - 1, i / l.sh);
        l.st_q0[i] = q0;
        l.st_n[i] = (q1 - q0 + 1) * l.cq;
        most = std::max(most, l.st_n[i]);
        if (i % l.sh == 0 && i / l.sh < l.q_rows) l.st_first |= 1u << i;
      }
      l.b_bytes = static_cast<uint32_t>(most) * 128;
    }
    l.stage_bytes = l.a_bytes + l.b_bytes;
    // stacked layers' stages are smaller: a deeper ring in a little more of the shared memory
    l.stages = std::min<int>(8, ((l.q_rows > 1 ? 216 : 200) * 1024) / l.stage_bytes);
    l.smem = 1024 + l.stages * l.stage_bytes + (2 * l.stages + 2 * kMaxAcc + 2) * 8 + 16 + 12 * y.cp + 64;
    if (h->int8 && (rc = upload_offsets(h, l, x.zero, colsum, y.cp))) return rc;
    if (h->int8) l.sat = round_first(h, l, x, y, scale, bias);
    // band mode where the layer's weights stay resident beside a ring of at least kh + 1 input
    // rows: every input row then crosses from L2 once a band instead of once a kernel row
    const int nt = round16(l.cout), chunks = x.cp * h->eb / 16, pairs = (chunks + 1) / 2;
    const uint32_t w_bytes = static_cast<uint32_t>(l.kh * l.kw * pairs * nt * 32);
    if (l.residual < 0 && l.kh <= 3 && l.kw <= 3 && (l.sw == 1 || l.sw == 2) && l.pl <= 2 && nt <= 256 &&
        w_bytes <= 160 * 1024 && !kNoBand) {
      const int fl = -((l.pl + l.sw - 1) / l.sw);  // floor(-pl / sw)
      int max_off = 0;
      for (int kx = 0; kx < l.kw; ++kx) {
        const int d = kx - l.pl - l.sw * fl;
        l.kx_parity[kx] = d % l.sw;
        l.kx_off[kx] = d / l.sw;
        max_off = std::max(max_off, l.kx_off[kx]);
      }
      const int plane_px = (128 + max_off + 7) / 8 * 8;
      const uint32_t slot_bytes = static_cast<uint32_t>(2 * pairs * l.sw * plane_px * 16);
      const uint32_t tail = (2 * 16 + 2 * kMaxAcc + 2) * 8 + 16 + 12 * y.cp + 64;
      const long long room = 232448 - 1024 - 1024 - static_cast<long long>(w_bytes) - tail;
      const int slots = static_cast<int>(std::min<long long>(16, room / slot_bytes));
      if (slots >= l.kh + 1) {
        l.band = true;
        l.pairs = pairs;
        l.band_chunks = chunks;
        l.plane_px = plane_px;
        l.band_rows = (y.h - 1) * l.sh + l.kh;
        l.gx0 = fl + 8;  // the tensor map's base is 8 pixel groups to the left (gap columns)
        l.slot_bytes = slot_bytes;
        l.load_bytes = static_cast<uint32_t>(chunks * l.sw * plane_px * 16);
        l.w_bytes = w_bytes;
        l.stages = slots;
        // row stacking as the other mode has it: q output rows a tile, each its own MMAs into its own
        // accumulator columns (N = q x cq), where q divides the output's height and q * cq <= 256
        // (a tile holds all the (q - 1) * sh + kh input rows it reads at once: the ring keeps one more)
        int q = 1;
        for (int k = 1; k <= y.h && k * nt <= 256; ++k)
          if (y.h % k == 0 && (k - 1) * l.sh + l.kh + 1 <= slots) q = k;
        l.q_rows = q;
        l.krows = 1;
        l.cq = nt;
        l.nt = q * nt;
        l.n_tiles = 1;
        l.smem = 1024 + w_bytes + slots * slot_bytes + (2 * slots + 2 * kMaxAcc + 2) * 8 + 16 + 12 * y.cp + 64;
        const std::vector<uint8_t> img = band_weight_image(h, l, nt);
        return upload(h, &l.wimg, img);
      }
    }
  }
  std::vector<uint8_t> img = weight_image(h, l, x.cp, l.nt, l.n_tiles, l.nkb);
  if (l.q_rows > 1) {
    // row stacking: input row i's blocks keep the weights of the output rows it serves only (the
    // others are zeros), in whole 16-row groups, so the swizzle holds
    std::vector<uint8_t> packed;
    for (int i = 0; i < l.krows; ++i) {
      const int q0 = l.st_q0[i], q1 = q0 + l.st_n[i] / l.cq - 1;
      l.st_off[i] = static_cast<uint32_t>(packed.size());
      for (int kb = 0; kb < l.nkb; ++kb) {
        const size_t pitch = kb == l.nkb - 1 ? static_cast<size_t>(l.tail) : 128;
        const uint8_t* blk = img.data() + static_cast<size_t>(i) * l.row_bytes + static_cast<size_t>(kb) * l.nt * 128;
        packed.insert(packed.end(), blk + static_cast<size_t>(q0) * l.cq * pitch, blk + static_cast<size_t>(q1 + 1) * l.cq * pitch);
      }
    }
    img.swap(packed);
  }
  if ((rc = upload(h, &l.wimg, img))) return rc;
  return CREC_OK;
}

int alloc_values(crec_handle* h) {
  for (size_t i = 0; i < h->v.size(); ++i) {
    Value& v = h->v[i];
    if (!v.real) continue;
    const long long cols = h->max_cols >> v.shift;
    v.pitch = cols * v.cp * h->eb;
    v.bytes = static_cast<size_t>(v.h + 2 * v.ph) * v.pitch + 2 * kGuard;
    CK(cudaMalloc(&v.alloc, v.bytes));
    CK(cudaMemset(v.alloc, h->int8 ? v.zero : 0, v.bytes));
    v.base = v.alloc + kGuard;
  }
  return CREC_OK;
}

int encode_map(crec_handle* h, CUtensorMap* m, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1,
               uint64_t s2, uint32_t inner = 128) {
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {s1, s2};
  const cuuint32_t box[3] = {inner, 128, 1};  // inner bytes (128, 64 or 32) in that width's swizzle
  const cuuint32_t es[3] = {1, 1, 1};
  const CUtensorMapSwizzle sw = inner == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                : inner == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                              : CU_TENSOR_MAP_SWIZZLE_32B;
  const CUresult r = h->encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, es,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(h, CREC_E_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
  return CREC_OK;
}

// A band-mode layer's input: (channel byte, pixel parity, pixel group, row), the base `base`; boxes
// of 16 channel bytes x plane_px groups of one parity and row.
int encode_map4(crec_handle* h, CUtensorMap* m, const void* base, uint64_t cbytes, uint64_t sw, uint64_t groups,
                uint64_t rows, uint64_t pitch, uint32_t plane_px) {
  const cuuint64_t dims[4] = {cbytes, sw, groups, rows};
  const cuuint64_t strides[3] = {cbytes, sw * cbytes, pitch};
  const cuuint32_t box[4] = {16, 1, plane_px, 1};
  const cuuint32_t es[4] = {1, 1, 1, 1};
  const CUresult r = h->encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(base), dims, strides, box, es,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(h, CREC_E_CUDA, "cuTensorMapEncodeTiled (4-d) failed (" + std::to_string(r) + ")");
  return CREC_OK;
}

// The crop kernel's shared memory for a run whose widest bucket is max_bw.
size_t crop_smem_bytes(const crec_handle* h, int max_bw) { return crop_smem(h->height, max_bw).total + 16; }
// crop_wide_kernel's shared memory, whatever the lines (one CTA an SM)
constexpr size_t kWideSmem = 200 << 10;

// Kernel kinds of the profile: 0 crop+stem, 1 dense convolutions (tcgen05), 2 depthwise, 3 head+CTC, 4 collapse.
enum ProfKind { kProfCrop = 0, kProfConv = 1, kProfDw = 2, kProfHead = 3, kProfCollapse = 4 };

// Brackets one launch with a pair of events when profiling (the pair's times are read after the call's sync).
struct ProfScope {
  crec_handle* h;
  int kind;
  cudaEvent_t end = nullptr;
  ProfScope(crec_handle* hh, int k, int layer) : h(hh), kind(k) {
    ++h->st_launches;
    if (!h->profile) return;
    if (h->ev_used + 2 > h->ev_pool.size()) {
      for (int i = 0; i < 64; ++i) {
        cudaEvent_t e;
        cudaEventCreate(&e);
        h->ev_pool.push_back(e);
      }
      h->ev_kind.resize(h->ev_pool.size() / 2);
      h->ev_layer.resize(h->ev_pool.size() / 2);
    }
    cudaEventRecord(h->ev_pool[h->ev_used], h->stream);
    end = h->ev_pool[h->ev_used + 1];
    h->ev_kind[h->ev_used / 2] = k;
    h->ev_layer[h->ev_used / 2] = layer;
    h->ev_used += 2;
  }
  ~ProfScope() {
    if (end) cudaEventRecord(end, h->stream);
  }
};

void collect_profile(crec_handle* h) {
  for (size_t i = 0; i + 1 < h->ev_used; i += 2) {
    float ms = 0;
    if (cudaEventElapsedTime(&ms, h->ev_pool[i], h->ev_pool[i + 1]) == cudaSuccess) {
      h->prof_ms[h->ev_kind[i / 2]] += ms;
      h->prof_count[h->ev_kind[i / 2]] += 1;
      const size_t li = static_cast<size_t>(h->ev_layer[i / 2]);
      if (li < h->lprof_ms.size()) {
        h->lprof_ms[li] += ms;
        h->lprof_count[li] += 1;
      }
    }
  }
  h->ev_used = 0;
}

// Algorithmic work of a run, by kernel kind: multiply-adds x 2 over the lines' own columns (gaps
// excluded; padded channels and K excluded), as the roofline counts it.
void add_run_ops(crec_handle* h, const int* bw, int a, int b) {
  if (!h->profile) return;
  long long width = 0;
  for (int i = a; i < b; ++i) width += bw[i];
  for (size_t li = 0; li < h->l.size(); ++li) {
    const Layer& l = h->l[li];
    if (l.kind == kKindResize) continue;
    const Value& y = h->v[l.out];
    const double pixels = static_cast<double>(y.h) * static_cast<double>(width >> y.shift);
    const double taps = l.kh * l.kw;
    const int kind = l.kind == kKindDw ? kProfDw : li == 0 ? kProfCrop : li + 1 == h->l.size() ? kProfHead : kProfConv;
    const double ops = 2.0 * pixels * taps * l.cout * (l.kind == kKindDw ? 1 : l.cin);
    h->prof_ops[kind] += ops;
    if (li < h->lprof_ops.size()) h->lprof_ops[li] += ops;
  }
}

// One dense convolution (layer li) over a run of `cols` input columns: its tensor maps, the
// conv_gemm_kernel launch on the handle's stream.
int launch_conv(crec_handle* h, size_t li, long long cols) {
  cudaStream_t s = h->stream;
  const Layer& l = h->l[li];
  const Value& x = h->v[l.in];
  const Value& y = h->v[l.out];
  const Value& xp = h->v[x.phys];
  const int oh = y.h;
  const long long ow = cols >> y.shift;
  ConvParams p{};
  const long long in_pitch = xp.pitch;
  const uint64_t px = static_cast<uint64_t>(x.cp) * h->eb;
  if (l.band) {
    const long long in_cols = cols >> x.shift;
    const uint8_t* base = xp.base - 8LL * l.sw * static_cast<long long>(px);
    int rc = encode_map4(h, &p.tmap[0], base, px, static_cast<uint64_t>(l.sw),
                         static_cast<uint64_t>(in_cols / l.sw + 8 + l.plane_px), static_cast<uint64_t>(x.h + 2 * xp.ph),
                         static_cast<uint64_t>(in_pitch), static_cast<uint32_t>(l.plane_px));
    if (rc) return rc;
    p.num_bands = static_cast<int>((ow + 127) / 128);
    p.band_rows = l.band_rows;
    p.kh = l.kh;
    p.kw = l.kw;
    p.sh = l.sh;
    p.sw = l.sw;
    p.pairs = l.pairs;
    p.chunks = l.band_chunks;
    p.plane_px = l.plane_px;
    p.gx0 = l.gx0;
    for (int k = 0; k < 3; ++k) {
      p.kx_parity[k] = l.kx_parity[k];
      p.kx_off[k] = l.kx_off[k];
    }
    p.slot_bytes = l.slot_bytes;
    p.load_bytes = l.load_bytes;
    p.w_bytes = l.w_bytes;
    p.row0 = xp.ph - l.pt;
    if (p.row0 < 0) return set_error(h, CREC_E_MODEL, "band mode: a padding wider than the input's border rows");
  }
  for (int i = 0; i < l.krows && !l.band; ++i) {  // input row i of a tile's group of q_rows output rows
    const uint8_t* base = xp.base + static_cast<long long>(i - l.pt + xp.ph) * in_pitch - static_cast<long long>(l.pl) * px;
    int rc = encode_map(h, &p.tmap[i], base, static_cast<uint64_t>(l.nkb) * 128, static_cast<uint64_t>(ow),
                        static_cast<uint64_t>(oh / l.q_rows), static_cast<uint64_t>(l.sw) * px,
                        static_cast<uint64_t>(l.q_rows) * l.sh * in_pitch);
    if (!rc && l.tail < 128)
      rc = encode_map(h, &p.tmap_tail[i], base, static_cast<uint64_t>(l.nkb) * 128, static_cast<uint64_t>(ow),
                      static_cast<uint64_t>(oh / l.q_rows), static_cast<uint64_t>(l.sw) * px,
                      static_cast<uint64_t>(l.q_rows) * l.sh * in_pitch, static_cast<uint32_t>(l.tail));
    if (rc) return rc;
  }
  p.tail_bytes = l.band ? 128 : l.tail;
  p.row_bytes = l.row_bytes;
  p.wimg = l.wimg;
  p.krows = l.krows;
  p.q_rows = l.q_rows;
  for (int i = 0; i < l.krows; ++i) {
    p.st_q0[i] = l.st_q0[i];
    p.st_n[i] = l.st_n[i];
    p.st_off[i] = l.st_off[i];
  }
  p.st_first = l.st_first;
  p.cq = l.cq;
  p.cq_inv = (65536 + l.cq / 16 - 1) / (l.cq / 16);
  p.nkb = l.nkb;
  p.last_steps = l.last_steps;
  p.nt = l.nt;
  p.n_tiles = l.n_tiles;
  p.oh = oh;
  p.ow = static_cast<int>(ow);
  p.m_per_row = static_cast<int>((ow + 127) / 128);
  p.num_tiles = (oh / l.q_rows) * p.m_per_row * l.n_tiles;
  p.nt_magic = div_magic(static_cast<uint32_t>(l.n_tiles));
  p.mpr_magic = div_magic(static_cast<uint32_t>(p.m_per_row));
  // the multiply-high divisions are exact for x * d < 2^32 (x a tile or column-block index)
  if (static_cast<unsigned long long>(p.num_tiles) * static_cast<unsigned>(std::max(l.n_tiles, p.m_per_row)) >= (1ull << 32))
    return set_error(h, CREC_E_RANGE, "a run with too many conv tiles");
  p.stages = l.stages;
  p.stage_bytes = l.stage_bytes;
  p.a_bytes = l.a_bytes;
  p.b_bytes = l.b_bytes;
  p.out = y.base;
  p.out_ph = y.ph;
  p.out_pitch = y.pitch;
  p.cp_out = y.cp;
  p.c_out = l.cout;
  p.ebytes = h->eb;
  p.off = l.hoff;
  p.scale = l.scale;
  p.bias = l.dbias;
  p.out_zero = y.zero;
  p.relu = l.relu;
  p.sat = l.sat;
  p.n_acc = conv_accumulators(l.nt);
  p.out_inv_scale = h->int8 ? 1.0f / y.scale : 1.0f;
  if (l.residual >= 0) {
    const Value& r = h->v[l.residual];
    const Value& rp = h->v[r.phys];
    p.res = rp.base;
    p.res_ph = rp.ph;
    p.res_cp = rp.cp;
    p.res_shift = rp.shift - y.shift;
    p.res_zero = r.zero;
    p.res_pitch = rp.pitch;
    p.res_scale = r.scale;
  }
  p.mask8 = h->d_mask;
  p.out_shift = y.shift;
  p.err = h->d_err;
  p.wait_ns = kWaitNs;
  if (h->inject_timeout) {  // test hook: this launch's loads never come, its waits end after 1 ms
    h->inject_timeout = false;
    p.wait_ns = 1000000ull;
    p.idle_producer = 1;
  }
  const int grid = std::min(l.band ? p.num_bands : p.num_tiles, h->sms);
  ProfScope prof(h, kProfConv, static_cast<int>(li));
  // the layer's compile-time form
  auto run = [&](auto int8, auto fast, auto res, auto sat, auto stack) -> int {
    constexpr bool kI8 = decltype(int8)::value, kF = decltype(fast)::value, kR = decltype(res)::value,
                   kS = decltype(sat)::value, kQ = decltype(stack)::value;
    // band mode has no residual
    auto* k = l.band ? conv_gemm_kernel<kI8, kF, false, kS, kQ, true> : conv_gemm_kernel<kI8, kF, kR, kS, kQ, false>;
    CK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, l.smem));
    k<<<grid, kConvThreads, l.smem, s>>>(p);
    return CREC_OK;
  };
  using T = std::true_type;
  using F = std::false_type;
  auto by_stack = [&](auto int8, auto fast, auto res, auto sat) {
    return l.q_rows > 1 ? run(int8, fast, res, sat, T{}) : run(int8, fast, res, sat, F{});
  };
  auto by_sat = [&](auto int8, auto fast, auto res) {
    return l.sat ? by_stack(int8, fast, res, T{}) : by_stack(int8, fast, res, F{});
  };
  auto by_res = [&](auto int8, auto fast) {
    return l.residual >= 0 ? by_sat(int8, fast, T{}) : by_sat(int8, fast, F{});
  };
  int rc;
  if (h->int8 && l.fast) rc = by_res(T{}, T{});
  else if (h->int8) rc = by_res(T{}, F{});
  else rc = l.residual >= 0 ? by_stack(F{}, F{}, T{}, F{}) : by_stack(F{}, F{}, F{}, F{});
  if (rc) return rc;
  CK(cudaGetLastError());
  return CREC_OK;
}

// The head (the last layer, a 1x1 convolution on one row) over `cols` input columns, fused with the
// frames' argmax and (INT8: in a kernel of its own after it) their CTC probabilities.
int launch_head(crec_handle* h, size_t li, long long cols) {
  cudaStream_t s = h->stream;
  const Layer& l = h->l[li];
  const Value& x = h->v[l.in];
  const Value& y = h->v[l.out];
  const Value& xp = h->v[x.phys];
  const long long ow = cols >> y.shift;
  HeadParams p{};
  // a frame's K bytes exactly: the last K block's box past them reads zeros (TMA's fill), not the
  // next frame's bytes
  int rc = encode_map(h, &p.tmap, xp.base + static_cast<long long>(xp.ph) * xp.pitch,
                      static_cast<uint64_t>(x.cp) * h->eb, static_cast<uint64_t>(ow), 1,
                      static_cast<uint64_t>(x.cp) * h->eb, static_cast<uint64_t>(xp.pitch));
  if (rc) return rc;
  p.wimg = l.wimg;
  p.nkb = l.nkb;
  p.last_steps = l.last_steps;
  p.classes = l.cout;
  p.nchunk = l.nchunk;
  p.chunks = l.chunks;
  p.ow = static_cast<int>(ow);
  p.num_tiles = static_cast<int>((ow + 127) / 128);
  p.a_bytes = l.a_bytes;
  p.b_bytes = l.b_bytes;
  p.off = l.hoff;
  p.scale = l.scale;
  p.bias = l.dbias;
  p.out_zero = y.zero;
  p.out_inv_scale = h->int8 ? 1.0f / y.scale : 1.0f;
  p.table = h->head_table;
  p.nb_codes = h->d_nb_codes;
  p.nb_row_bytes = h->nb_row_bytes;
  p.nb_frame = h->d_nb_frame;
  p.nb_best = h->d_nb_best;
  p.nb_count = h->d_nb_count;
  p.mask8 = h->d_mask;
  p.out_shift = y.shift;
  p.frame_id = h->d_frame_id;
  p.frame_prob = h->d_frame_prob;
  p.logits = h->d_logits;
  p.err = h->d_err;
  p.sat = l.sat ? 1 : 0;
  const int grid = std::min(p.num_tiles, h->sms);
  p.nb_region = (p.num_tiles + grid - 1) / grid * 128;
  ProfScope prof(h, kProfHead, static_cast<int>(li));
  auto launch = [&](auto* k) -> int {
    CK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, l.smem));
    k<<<grid, kHeadThreads, l.smem, s>>>(p);
    return CREC_OK;
  };
  const int lrc = !h->int8            ? launch(head_ctc_kernel<false, false, false>)
                  : l.fast && l.sat   ? launch(head_ctc_kernel<true, true, true>)
                  : l.fast            ? launch(head_ctc_kernel<true, true, false>)
                  : l.sat             ? launch(head_ctc_kernel<true, false, true>)
                                      : launch(head_ctc_kernel<true, false, false>);
  if (lrc) return lrc;
  CK(cudaGetLastError());
  if (h->int8) {  // the listed frames' class-order sums
    ProfScope sums(h, kProfHead, static_cast<int>(li));
    const int smem = kSumRows * kSumPitch * static_cast<int>(sizeof(float));
    CK(cudaFuncSetAttribute(ctc_sums_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    ctc_sums_kernel<<<grid, kSumThreads, smem, s>>>(h->d_nb_codes, h->nb_row_bytes, h->d_nb_frame, h->d_nb_best,
                                                    h->d_nb_count, p.nb_region, h->ctc_terms, l.cout, h->d_frame_prob);
    CK(cudaGetLastError());
  }
  return CREC_OK;
}

// Launches every layer for the lines laid out in h_lines (already on the device), `cols` input columns.
int launch_run(crec_handle* h, int n, long long cols, bool keep_crops) {
  cudaStream_t s = h->stream;
  const Layer& stem = h->l[0];
  const Value& x0 = h->v[h->inp];
  const Value& s0 = h->v[stem.out];
  {
    CropParams p{};
    p.pages = h->d_pages;
    p.lines = h->d_lines;
    p.n = n;
    p.height = h->height;
    p.flip_margin = h->cfg.crop.flip_margin;
    p.flip_needs_dark = h->cfg.crop.flip_needs_dark;
    p.crops_out = keep_crops ? h->d_crops : nullptr;
    p.crops_pitch = h->crops_pitch;
    p.crops_in = h->run_crops;
    p.crops_in_pitch = h->crops_in_pitch;
    p.kh = stem.kh;
    p.kw = stem.kw;
    p.sh = stem.sh;
    p.sw = stem.sw;
    p.pt = stem.pt;
    p.pl = stem.pl;
    p.cout = stem.cout;
    p.cp_out = s0.cp;
    p.w8 = stem.dw8;
    p.wf = stem.dwf;
    p.scale = stem.scale;
    p.bias = stem.dbias;
    p.colsum = stem.colsum;
    p.in_table = h->in_table;
    p.in_zero = x0.zero;
    p.out_zero = s0.zero;
    p.relu = stem.relu;
    p.sat = stem.sat;
    p.out_inv_scale = h->int8 ? 1.0f / s0.scale : 1.0f;
    p.out = s0.base;
    p.out_ph = s0.ph;
    p.out_pitch = s0.pitch;
    p.out_shift = s0.shift;
    p.err = h->d_err;
    p.claim = h->d_claim;
    p.order = h->d_order;
    p.wide = h->d_wide;
    p.wide_pitch = h->cfg.max_width;
    int max_bw = 8;
    for (int i = 0; i < n; ++i) max_bw = std::max(max_bw, h->run_bw[i]);
    p.max_bw = max_bw;
    const size_t smem = crop_smem_bytes(h, max_bw);
    ProfScope prof(h, kProfCrop, 0);
    if (h->run_wide > 0 && !h->run_crops) {
      // the lines beyond the crop kernel's reach first, into their raw crops
      WideParams w{};
      w.pages = h->d_pages;
      w.lines = h->d_lines;
      w.index = h->d_wide_idx;
      w.height = h->height;
      w.vtaps = h->run_vtaps;
      w.htaps = h->run_htaps;
      w.out = h->d_wide;
      w.pitch = h->cfg.max_width;
      w.err = h->d_err;
      // 64 columns of coefficients a strip where they fit; the intermediate takes the rest of
      // kWideSmem, and must hold one column of the tallest span
      w.hk_cols = std::max(1, std::min(64, static_cast<int>(kWideSmem / 4 / static_cast<size_t>(4 * (w.htaps + 2)))));
      const size_t fixed = wide_smem(w.height, w.vtaps, w.htaps, w.hk_cols, 0);
      if (fixed >= kWideSmem || kWideSmem - fixed < static_cast<size_t>(h->run_rows))
        return set_error(h, CREC_E_RANGE, "a line's source span (" + std::to_string(h->run_rows) + " rows, " +
                                              std::to_string(std::max(w.vtaps, w.htaps)) +
                                              " taps) beyond the resampler's shared memory");
      w.tmp_bytes = static_cast<int>(kWideSmem - fixed) & ~15;
      CK(cudaFuncSetAttribute(crop_wide_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kWideSmem)));
      crop_wide_kernel<<<h->run_wide, kCropThreads, kWideSmem, s>>>(w);
      CK(cudaGetLastError());
      ++h->st_launches;  // timed with the crop's
    }
    // persistent: as many CTAs as fit at once (each takes lines until none are left)
    auto launch = [&](auto* k) -> int {
      // the attribute is the function's, for every handle in the process: set it for this one's size
      CK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
      int per_sm = 0;
      CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kCropThreads, smem));
      const int grid = std::min(n, std::max(1, per_sm) * h->sms);
      k<<<grid, kCropThreads, smem, s>>>(p);
      return CREC_OK;
    };
    const int lrc = h->int8 ? launch(crop_stem_kernel<true>) : launch(crop_stem_kernel<false>);
    if (lrc) return lrc;
    CK(cudaGetLastError());
  }
  for (size_t li = 1; li < h->l.size(); ++li) {
    const Layer& l = h->l[li];
    if (l.kind == kKindResize) continue;
    const Value& x = h->v[l.in];
    const Value& y = h->v[l.out];
    const Value& xp = h->v[x.phys];
    const int oh = y.h;
    const long long ow = cols >> y.shift;
    if (li + 1 == h->l.size()) {
      const int rc = launch_head(h, li, cols);
      if (rc) return rc;
      continue;
    }
    if (l.kind == kKindDw) {
      DwParams p{};
      p.in = xp.base;
      p.in_ph = xp.ph;
      p.in_cp = xp.cp;
      p.in_shift = x.extra;
      p.in_zero = x.zero;
      p.in_pitch = xp.pitch;
      p.kh = l.kh;
      p.kw = l.kw;
      p.pt = l.pt;
      p.pl = l.pl;
      p.oh = oh;
      p.ow = static_cast<int>(ow);
      p.c = l.cout;
      p.cp = y.cp;
      p.w8 = l.dw8;
      p.wf = l.dwf;
      p.scale = l.scale;
      p.bias = l.dbias;
      p.out_zero = y.zero;
      p.relu = l.relu;
      p.sat = l.sat ? 1 : 0;
      p.out_inv_scale = h->int8 ? 1.0f / y.scale : 1.0f;
      p.out = y.base;
      p.out_ph = y.ph;
      p.out_pitch = y.pitch;
      p.mask8 = h->d_mask;
      p.out_shift = y.shift;
      p.wt = l.dwt;
      p.dwc = l.dwc;
      p.g_magic = div_magic(static_cast<uint32_t>(y.cp / 16));
      ProfScope prof(h, kProfDw, static_cast<int>(li));
      if (h->int8 && l.dwt) {
        const long long tiles = static_cast<long long>(oh) * ((ow + kDwTile - 1) / kDwTile);
        const int ncols = dw_row_cols(l.kw, x.extra);
        const int smem = ((ncols * y.cp + 15) & ~15) + 24 * y.cp;
        auto* k = l.sat ? dw_row_kernel<true> : dw_row_kernel<false>;
        CK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        k<<<static_cast<int>(tiles), 256, smem, s>>>(p);
      } else if (!h->int8 && l.kh == 1 && xp.cp == y.cp && (l.kw == 3 || l.kw == 5 || l.kw == 7 || l.kw == 9)) {
        // FP16, one kernel row: a CTA 2 x kDwF16Run output pixels of a row
        const int tiles = static_cast<int>(static_cast<long long>(oh) * ((ow + 2 * kDwF16Run - 1) / (2 * kDwF16Run)));
        if (l.kw == 3) dw_row_f16_kernel<3><<<tiles, 256, 0, s>>>(p);
        else if (l.kw == 5) dw_row_f16_kernel<5><<<tiles, 256, 0, s>>>(p);
        else if (l.kw == 7) dw_row_f16_kernel<7><<<tiles, 256, 0, s>>>(p);
        else dw_row_f16_kernel<9><<<tiles, 256, 0, s>>>(p);
      } else {
        const long long total = static_cast<long long>(oh) * ow * (y.cp / 16);
        const int grid = static_cast<int>((total + 255) / 256);
        if (h->int8)
          dw_kernel<true><<<grid, 256, 0, s>>>(p);
        else
          dw_kernel<false><<<grid, 256, 0, s>>>(p);
      }
      CK(cudaGetLastError());
      continue;
    }
    if (int rc = launch_conv(h, li, cols)) return rc;
  }
  CollapseParams c{};
  c.frame_id = h->d_frame_id;
  c.frame_prob = h->d_frame_prob;
  c.line_frame0 = h->d_frame0;
  c.length = h->d_length;
  c.n = n;
  c.count = h->d_count;
  c.ids = h->d_ids;
  c.frames = h->d_frames;
  c.probs = h->d_probs;
  {
    ProfScope prof(h, kProfCollapse, static_cast<int>(h->l.size()));
    collapse_kernel<<<(n + 127) / 128, 128, 0, s>>>(c);
  }
  CK(cudaGetLastError());
  return CREC_OK;
}

// Host staging for one call (pinned, grown on demand, never shrunk): each run of a call has its
// own slices, so every run's copies and launches are queued at once and the call syncs once.
template <class T>
int grow_pinned(crec_handle* h, T** p, size_t* cap, size_t need) {
  if (need <= *cap) return CREC_OK;
  const size_t n = std::max(need, *cap * 2);
  cudaFreeHost(*p);
  *p = nullptr;
  *cap = 0;
  CK(cudaHostAlloc(reinterpret_cast<void**>(p), n * sizeof(T), cudaHostAllocDefault));
  *cap = n;
  return CREC_OK;
}

template <class T>
int grow_device(crec_handle* h, T** p, size_t* cap, size_t need) {
  if (need <= *cap) return CREC_OK;
  const size_t n = std::max(need, *cap * 2);
  CK(cudaStreamSynchronize(h->stream));  // nothing queued may still use the old buffer
  cudaFree(*p);
  *p = nullptr;
  *cap = 0;
  CK(cudaMalloc(reinterpret_cast<void**>(p), n * sizeof(T)));
  *cap = n;
  return CREC_OK;
}

struct Source {  // where a call's lines come from
  const int32_t* page_of = nullptr;
  const crec_box* boxes = nullptr;
  const uint8_t* crops = nullptr;  // ready crops, [n][height][pitch]
  int pitch = 0;
  const int32_t* widths = nullptr;
};

// Lays out lines [a, b) of a call as one run (its LineDescs, mask, frame starts and lengths, claim
// keys in the call's staging at the given offsets); returns the run's input columns in *cols.
// The segments are one prefix sum; each line's crop region, checks, descriptor and mask bytes are
// then independent, so they run on the host pool in parts of consecutive lines, and the first
// failing line's error is the one reported, as one pass in line order would.
int layout_run(crec_handle* h, const Source& src, const int* bw, int a, int b, size_t mask_off, long long* cols_out) {
  const crec_crop_rule& rule = h->cfg.crop;
  long long seg = h->gap;
  for (int i = a; i < b; ++i) {
    h->hs_lines[i].seg = static_cast<int>(seg);
    seg += bw[i] + h->gap;
  }
  const long long end = seg - h->gap;  // the column after the last line
  const long long cols = round_up(seg, 128LL << h->max_shift);
  uint8_t* mask = h->hs_mask + mask_off;
  const int gap8 = h->gap / 8;
  struct Part {
    int err = CREC_OK;
    std::string msg;
    std::vector<int> wide;  // lines past the crop kernel's reach, in line order
    int ht = 0, vt = 0, rows = 0;
  };
  const int m = b - a;
  const int parts = h->pool && m >= kPoolLines ? std::min(4 * h->pool->threads(), m / 256) : 1;
  std::vector<Part> part(static_cast<size_t>(parts));
  auto lay = [&](int p) {
    const int lo = a + static_cast<int>(static_cast<long long>(m) * p / parts);
    const int hi = a + static_cast<int>(static_cast<long long>(m) * (p + 1) / parts);
    Part& P = part[static_cast<size_t>(p)];
    for (int i = lo; i < hi; ++i) {
      LineDesc& d = h->hs_lines[i];
      d.wide = -1;
      double reg[4] = {0, 0, 1, 1};
      int width = 0;
      if (src.crops) {
        width = src.widths[i];
        if (width <= 0 || width > bw[i] || bw[i] > src.pitch) {
          P.err = CREC_E_RANGE;
          P.msg = "recognize_crops: line " + std::to_string(i) + " width " + std::to_string(width) + ", bucket " +
                  std::to_string(bw[i]);
          return;
        }
        d.page = 0;
      } else {
        crec_crop_region(&src.boxes[i], &rule, reg, &width);
        const int pg = src.page_of[i];
        if (pg < 0 || pg >= static_cast<int>(h->pages.size())) {
          P.err = CREC_E_INVALID;
          P.msg = "line " + std::to_string(i) + ": page " + std::to_string(pg) + " not set";
          return;
        }
        if (width > bw[i]) {
          P.err = CREC_E_RANGE;
          P.msg = "crop_lines: line " + std::to_string(i) + " is " + std::to_string(width) + " px wide, the batch " +
                  std::to_string(bw[i]);
          return;
        }
        // the crop kernel's reach: at most kMaxTaps taps a sample (PIL's ksize, 2 ceil(support) + 1)
        // and kMaxSrcRows source rows (the bound the kernel computes); past it, crop_wide_kernel
        const double sx = std::max(1.0, (reg[2] - reg[0]) / width), sy = std::max(1.0, (reg[3] - reg[1]) / rule.height);
        if (!(sx < 1e6) || !(sy < 1e6)) {
          P.err = CREC_E_RANGE;
          P.msg = "line " + std::to_string(i) + ": a degenerate crop region";
          return;
        }
        const int ht = static_cast<int>(std::ceil(sx)) * 2 + 1, vt = static_cast<int>(std::ceil(sy)) * 2 + 1;
        const int rows = static_cast<int>(std::ceil((reg[3] - reg[1]) + 2.0 * sy)) + 4;
        if (ht > kMaxTaps || vt > kMaxTaps || rows > kMaxSrcRows) {
          P.wide.push_back(i);
          P.ht = std::max(P.ht, ht);
          P.vt = std::max(P.vt, vt);
          P.rows = std::max(P.rows, rows);
        }
        d.page = pg;
      }
      d.x0 = reg[0];
      d.y0 = reg[1];
      d.x1 = reg[2];
      d.y1 = reg[3];
      d.width = width;
      d.bw = bw[i];
      d.next_seg = i + 1 < b ? h->hs_lines[i + 1].seg : static_cast<int>(cols);
      h->hs_frame0[i] = d.seg >> h->head_shift;
      h->hs_length[i] = std::min(bw[i] >> h->head_shift, width / rule.frame_px);
      // the claim order's key: a line's source width plus twice its bucket width, in buckets of 64
      // (the horizontal pass reads the one; the vertical pass, finish and stem work over the other)
      const double k = ((d.x1 - d.x0) + 2.0 * d.bw) / 64.0;
      h->hs_key[i] = kOrderBuckets - 1 - static_cast<int>(std::min<double>(kOrderBuckets - 1, std::max(0.0, k)));
      std::memset(mask + (d.seg / 8 - gap8), 0, static_cast<size_t>(gap8));
      std::memset(mask + d.seg / 8, 1, static_cast<size_t>(bw[i] / 8));
    }
  };
  if (parts > 1)
    h->pool->run(parts, lay);
  else
    lay(0);
  for (const Part& P : part)
    if (P.err) return set_error(h, P.err, P.msg);
  h->run_wide = h->run_vtaps = h->run_htaps = h->run_rows = 0;
  for (const Part& P : part) {
    for (int i : P.wide) {
      h->hs_lines[i].wide = h->run_wide;
      h->hs_wide[a + h->run_wide++] = i - a;
    }
    h->run_htaps = std::max(h->run_htaps, P.ht);
    h->run_vtaps = std::max(h->run_vtaps, P.vt);
    h->run_rows = std::max(h->run_rows, P.rows);
  }
  if (cols > h->max_cols) return set_error(h, CREC_E_RANGE, "a run wider than the configured columns");
  std::memset(mask + end / 8, 0, static_cast<size_t>((cols - end) / 8));
  *cols_out = cols;
  return CREC_OK;
}

// The crop kernel's claim order for lines [a, b) of the call (laid out): the costliest first, by
// a counting sort on the keys layout_run computed.
void order_run(crec_handle* h, int a, int b) {
  std::vector<int>& cnt = h->order_count;
  cnt.assign(kOrderBuckets + 1, 0);
  const int* key = h->hs_key.data();
  for (int i = a; i < b; ++i) ++cnt[key[i] + 1];
  for (int k = 0; k < kOrderBuckets; ++k) cnt[k + 1] += cnt[k];
  for (int i = a; i < b; ++i) h->hs_order[a + cnt[key[i]]++] = i - a;
}

// Lines [0, n) of a call, bucket widths bw[i]: cut into runs of at most max_lines lines and
// max_columns columns, each run laid out and queued while the one before computes; a finished
// run's decodings are read back while the next one computes; the last run's after one sync.
int recognize_all(crec_handle* h, const Source& src, const int* bw, int n, crec_lines* out) {
  out->total = 0;
  h->last_n = 0;  // until this call's last run is queued: no candidates from an earlier call
  if (n == 0) return CREC_OK;
  struct Run {
    int a, b;
    long long cols;
    size_t mask_off, frame_off;
  };
  std::vector<Run> runs;
  size_t mask_total = 0, frame_total = 0;
  const long long unit = 128LL << h->max_shift;
  const long long fit = h->max_cols / unit * unit;  // round_up(c, unit) <= max_cols exactly when c <= fit
  for (int a = 0; a < n;) {
    long long cols = h->gap;
    int b = a;
    while (b < n && b - a < h->cfg.max_lines) {
      const long long next = cols + bw[b] + h->gap;
      if (next > fit) break;
      cols = next;
      ++b;
    }
    if (b == a) return set_error(h, CREC_E_RANGE, "a line wider than the configured columns");
    const long long rc = round_up(cols, unit);
    runs.push_back({a, b, rc, mask_total, frame_total});
    mask_total += static_cast<size_t>(rc / 8);
    frame_total += static_cast<size_t>(rc >> h->head_shift);
    a = b;
  }
  int rc;
  size_t cap_dp_lines = h->cap_dp_lines, cap_dp_chars = h->cap_dp_chars, cap_dp_a = cap_dp_lines,
         cap_dp_c = cap_dp_chars, cap_dp_d = cap_dp_chars;
  if ((rc = grow_pinned(h, &h->hs_lines, &h->cap_lines, n)) || (rc = grow_pinned(h, &h->hs_frame0, &h->cap_frame0, n)) ||
      (rc = grow_pinned(h, &h->hs_length, &h->cap_length, n)) ||
      (rc = grow_pinned(h, &h->hs_mask, &h->cap_mask, mask_total)) ||
      (rc = grow_pinned(h, &h->hs_wide, &h->cap_hs_wide, n)) ||
      (rc = grow_pinned(h, &h->hs_order, &h->cap_hs_order, n)) ||
      (rc = grow_pinned(h, &h->h_run_total, &h->cap_run_total, runs.size())) ||
      (rc = grow_device(h, &h->dp_counts, &cap_dp_lines, n)) || (rc = grow_device(h, &h->dp_offsets, &cap_dp_a, n)) ||
      (rc = grow_device(h, &h->dp_ids, &cap_dp_chars, frame_total)) ||
      (rc = grow_device(h, &h->dp_frames, &cap_dp_c, frame_total)) ||
      (rc = grow_device(h, &h->dp_probs, &cap_dp_d, frame_total)))
    return rc;
  h->cap_dp_lines = std::min(cap_dp_lines, cap_dp_a);
  h->cap_dp_chars = std::min({cap_dp_chars, cap_dp_c, cap_dp_d});
  if (h->hs_key.size() < static_cast<size_t>(n)) h->hs_key.resize(static_cast<size_t>(n));
  if (!h->pool && n >= kPoolLines) {
    const int hw = static_cast<int>(std::thread::hardware_concurrency());
    h->pool = std::make_unique<crec::HostPool>(std::clamp(hw / 2, 1, 8) - 1);
  }
  while (h->ev_run.size() + 1 < runs.size()) {
    cudaEvent_t e = nullptr;
    CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    h->ev_run.push_back(e);
  }
  if (runs.size() > 1 && !h->read_stream) CK(cudaStreamCreateWithFlags(&h->read_stream, cudaStreamNonBlocking));
  cudaStream_t s = h->stream;
  h->st_runs = static_cast<long long>(runs.size());
  h->st_wide = 0;
  h->st_launches = 0;
  h->st_h2d = 0;
  h->st_d2h = 4 + 8;  // the error word, the total
  CK(cudaMemsetAsync(h->d_err, 0, sizeof(int), s));
  CK(cudaMemsetAsync(h->d_total, 0, sizeof(long long), s));
  // a finished run's decodings into the caller's buffers: its lines' counts and offsets, and the
  // characters the runs before it did not have (the call's total after it is `total`)
  long long read_total = 0;
  auto read_run = [&](const Run& q, long long total, cudaStream_t rs) -> int {
    if (total > out->capacity) return set_error(h, CREC_E_RANGE, "crec_lines: capacity too small");
    const size_t m = static_cast<size_t>(q.b - q.a);
    CK(cudaMemcpyAsync(out->counts + q.a, h->dp_counts + q.a, sizeof(int32_t) * m, cudaMemcpyDeviceToHost, rs));
    CK(cudaMemcpyAsync(out->offsets + q.a, h->dp_offsets + q.a, sizeof(int32_t) * m, cudaMemcpyDeviceToHost, rs));
    if (total > read_total) {  // the characters themselves, and nothing else
      const size_t k = static_cast<size_t>(total - read_total);
      CK(cudaMemcpyAsync(out->ids + read_total, h->dp_ids + read_total, sizeof(int32_t) * k, cudaMemcpyDeviceToHost, rs));
      CK(cudaMemcpyAsync(out->frames + read_total, h->dp_frames + read_total, sizeof(int32_t) * k,
                         cudaMemcpyDeviceToHost, rs));
      CK(cudaMemcpyAsync(out->probs + read_total, h->dp_probs + read_total, sizeof(float) * k, cudaMemcpyDeviceToHost,
                         rs));
    }
    CK(cudaStreamSynchronize(rs));
    read_total = total;
    return CREC_OK;
  };
  for (size_t r = 0; r < runs.size(); ++r) {
    const Run& q = runs[r];
    long long cols = 0;
    if ((rc = layout_run(h, src, bw, q.a, q.b, q.mask_off, &cols))) return rc;
    const int m = q.b - q.a;
    order_run(h, q.a, q.b);
    CK(cudaMemcpyAsync(h->d_order, h->hs_order + q.a, sizeof(int) * m, cudaMemcpyHostToDevice, s));
    h->st_h2d += static_cast<long long>(sizeof(int)) * m;
    if (h->run_wide > 0) {
      const size_t need = static_cast<size_t>(h->run_wide) * h->height * h->cfg.max_width;
      if ((rc = grow_device(h, &h->d_wide, &h->cap_wide, need))) return rc;
      CK(cudaMemcpyAsync(h->d_wide_idx, h->hs_wide + q.a, sizeof(int) * h->run_wide, cudaMemcpyHostToDevice, s));
      h->st_h2d += static_cast<long long>(sizeof(int)) * h->run_wide;
      h->st_wide += h->run_wide;
    }
    CK(cudaMemcpyAsync(h->d_lines, h->hs_lines + q.a, sizeof(LineDesc) * m, cudaMemcpyHostToDevice, s));
    CK(cudaMemcpyAsync(h->d_mask, h->hs_mask + q.mask_off, static_cast<size_t>(cols / 8), cudaMemcpyHostToDevice, s));
    CK(cudaMemcpyAsync(h->d_frame0, h->hs_frame0 + q.a, sizeof(int) * m, cudaMemcpyHostToDevice, s));
    CK(cudaMemcpyAsync(h->d_length, h->hs_length + q.a, sizeof(int) * m, cudaMemcpyHostToDevice, s));
    h->run_crops = nullptr;
    if (src.crops) {
      CK(cudaMemcpyAsync(h->d_crops_in, src.crops + static_cast<size_t>(q.a) * h->height * src.pitch,
                         static_cast<size_t>(m) * h->height * src.pitch, cudaMemcpyHostToDevice, s));
      h->run_crops = h->d_crops_in;
      h->crops_in_pitch = src.pitch;
    }
    h->st_h2d += static_cast<long long>(sizeof(LineDesc) * m + cols / 8 + 2 * sizeof(int) * m);
    if (src.crops) h->st_h2d += static_cast<long long>(m) * h->height * src.pitch;
    add_run_ops(h, bw, q.a, q.b);
    h->run_bw = bw + q.a;
    if ((rc = launch_run(h, m, cols, h->d_crops != nullptr))) return rc;
    {  // this run's characters packed after the previous runs'
      ProfScope prof(h, kProfCollapse, static_cast<int>(h->l.size()));
      scan_counts_kernel<<<1, 1024, 0, s>>>(h->d_count, m, h->dp_counts + q.a, h->dp_offsets + q.a, h->d_total);
      pack_kernel<<<(m * 32 + 255) / 256, 256, 0, s>>>(h->d_ids, h->d_frames, h->d_probs, h->d_frame0,
                                                      h->dp_counts + q.a, h->dp_offsets + q.a, m, h->dp_ids,
                                                      h->dp_frames, h->dp_probs);
      ++h->st_launches;
    }
    CK(cudaGetLastError());
    if (r + 1 < runs.size()) {  // the call's total after this run, and the run's end
      CK(cudaMemcpyAsync(h->h_run_total + r, h->d_total, sizeof(long long), cudaMemcpyDeviceToHost, s));
      CK(cudaEventRecord(h->ev_run[r], s));
      h->st_d2h += 8;
    }
    if (r > 0) {  // the run before this one, read back while this one computes
      CK(cudaEventSynchronize(h->ev_run[r - 1]));
      if ((rc = read_run(runs[r - 1], h->h_run_total[r - 1], h->read_stream))) return rc;
    }
  }
  CK(cudaMemcpyAsync(h->h_err, h->d_err, sizeof(int), cudaMemcpyDeviceToHost, s));
  CK(cudaMemcpyAsync(h->h_total, h->d_total, sizeof(long long), cudaMemcpyDeviceToHost, s));
  CK(cudaStreamSynchronize(s));
  if (h->inject_sticky) {  // test hook: the completion check fails as after a faulted kernel
    h->inject_sticky = false;
    CK(cudaErrorLaunchFailure);
  }
  if (h->profile) collect_profile(h);
  if (*h->h_err == kErrBadShape)
    return set_error(h, CREC_E_RANGE, "a line's crop beyond the resamplers' reach");
  if (*h->h_err)
    return set_error(h, CREC_E_TIMEOUT, "a kernel's bounded wait ran out (device error " + std::to_string(*h->h_err) + ")");
  const long long total = *h->h_total;
  if ((rc = read_run(runs.back(), total, s))) return rc;
  h->st_d2h += static_cast<long long>(8 * n + 12 * total);
  h->tot_h2d += h->st_h2d;
  h->tot_d2h += h->st_d2h;
  std::memcpy(out->lengths, h->hs_length, sizeof(int32_t) * n);
  out->total = total;
  const Run& last = runs.back();
  h->last_n = last.b - last.a;
  h->last_a = last.a;
  h->last_frame0.assign(h->hs_frame0 + last.a, h->hs_frame0 + last.b);
  h->last_len.assign(h->hs_length + last.a, h->hs_length + last.b);
  h->last_cols = last.cols;
  h->last_seg.resize(h->last_n);
  h->last_bw.resize(h->last_n);
  for (int i = last.a; i < last.b; ++i) {
    h->last_seg[i - last.a] = h->hs_lines[i].seg;
    h->last_bw[i - last.a] = h->hs_lines[i].bw;
  }
  return CREC_OK;
}

void free_all(crec_handle* h) {
  for (auto& v : h->v) cudaFree(v.alloc);
  for (auto& l : h->l) {
    cudaFree(l.wimg);
    cudaFree(l.colsum);
    cudaFree(l.scale);
    cudaFree(l.dbias);
    cudaFree(l.dw8);
    cudaFree(l.dwf);
    cudaFree(l.hoff);
    cudaFree(l.dwt);
    cudaFree(l.dwc);
  }
  cudaFree(h->in_table);
  cudaFree(h->head_table);
  cudaFree(h->ctc_terms);
  cudaFree(h->d_nb_codes);
  cudaFree(h->d_nb_frame);
  cudaFree(h->d_nb_best);
  cudaFree(h->d_nb_count);
  for (auto& sl : h->slot) {
    cudaFree(sl.mem);
    cudaFree(sl.d_pages);
    if (sl.done) cudaEventDestroy(sl.done);
    if (sl.unused) cudaEventDestroy(sl.unused);
  }
  cudaFree(h->d_ext_pages);
  if (h->copy_stream) cudaStreamDestroy(h->copy_stream);
  cudaFree(h->d_lines);
  cudaFree(h->d_mask);
  cudaFree(h->d_frame0);
  cudaFree(h->d_length);
  cudaFree(h->d_frame_id);
  cudaFree(h->d_frame_prob);
  cudaFree(h->d_count);
  cudaFree(h->d_ids);
  cudaFree(h->d_frames);
  cudaFree(h->d_probs);
  cudaFree(h->d_err);
  cudaFree(h->d_crops);
  cudaFree(h->d_crops_in);
  cudaFree(h->d_claim);
  cudaFree(h->d_order);
  cudaFreeHost(h->hs_order);
  cudaFree(h->d_cand_cols);
  cudaFree(h->d_cand_ids);
  cudaFree(h->d_cand_vals);
  cudaFree(h->d_cand_fr);
  cudaFree(h->d_wide_idx);
  cudaFree(h->d_wide);
  cudaFreeHost(h->hs_wide);
  cudaFree(h->d_logits);
  cudaFreeHost(h->hs_lines);
  cudaFreeHost(h->hs_frame0);
  cudaFreeHost(h->hs_length);
  cudaFreeHost(h->hs_mask);
  cudaFreeHost(h->h_total);
  cudaFreeHost(h->h_run_total);
  for (cudaEvent_t e : h->ev_run) cudaEventDestroy(e);
  if (h->read_stream) cudaStreamDestroy(h->read_stream);
  h->pool.reset();
  cudaFree(h->dp_counts);
  cudaFree(h->dp_offsets);
  cudaFree(h->dp_ids);
  cudaFree(h->dp_frames);
  cudaFree(h->dp_probs);
  cudaFree(h->d_total);
  cudaFreeHost(h->h_err);
  for (cudaEvent_t e : h->ev_pool) cudaEventDestroy(e);
  if (h->stream) cudaStreamDestroy(h->stream);
}

int open_impl(crec_handle* h, const crec_config* c) {
  h->cfg = *c;
  if (c->precision != CREC_INT8 && c->precision != CREC_FP16) return set_error(h, CREC_E_INVALID, "precision");
  if (c->max_lines <= 0 || c->max_width <= 0 || c->max_width > 4096 || c->max_width % 8)
    return set_error(h, CREC_E_INVALID, "max_lines / max_width");
  if (c->crop.height <= 0 || c->crop.height > 64 || c->crop.frame_px <= 0 || c->crop.width_step <= 0)
    return set_error(h, CREC_E_INVALID, "crop rule");
  h->int8 = c->precision == CREC_INT8;
  h->eb = h->int8 ? 1 : 2;
  h->device = c->device;
  int count = 0;
  CK(cudaGetDeviceCount(&count));
  if (c->device < 0 || c->device >= count) return set_error(h, CREC_E_INVALID, "no CUDA device " + std::to_string(c->device));
  CK(cudaSetDevice(c->device));
  cudaDeviceProp prop{};
  CK(cudaGetDeviceProperties(&prop, c->device));
  if (prop.major != 10) return set_error(h, CREC_E_INVALID, std::string("this build runs on sm_100 (B200); device is ") + prop.name);
  h->sms = prop.multiProcessorCount;
  cudaDriverEntryPointQueryResult q{};
  void* fn = nullptr;
  CK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
  if (!fn || q != cudaDriverEntryPointSuccess) return set_error(h, CREC_E_CUDA, "cuTensorMapEncodeTiled is not available");
  h->encode = reinterpret_cast<EncodeTiled>(fn);
  CK(cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking));
  int rc = read_model(h, static_cast<const uint8_t*>(c->model), c->model_bytes);
  if (rc) return rc;
  if (h->height != c->crop.height) return set_error(h, CREC_E_MODEL, "the model reads crops of another height");
  if ((rc = plan_model(h))) return rc;
  if (c->crop.width_step % (1 << h->max_shift)) return set_error(h, CREC_E_MODEL, "crop width step and the network's stride");
  const long long per_line = c->max_width + h->gap;
  h->max_cols = c->max_columns > 0 ? c->max_columns : static_cast<long long>(c->max_lines) * per_line + h->gap;
  h->max_cols = round_up(h->max_cols, 128LL << h->max_shift);
  for (size_t i = 0; i < h->l.size(); ++i)
    if ((rc = setup_layer(h, i))) return rc;
  if ((rc = alloc_values(h))) return rc;
  if (h->int8) {
    std::vector<uint8_t> t(256);
    const Value& x = h->v[h->inp];
    for (int p = 0; p < 256; ++p) t[p] = quantize_in(1.0f - static_cast<float>(p) / 255.0f, x.scale, x.zero);
    if ((rc = upload(h, &h->in_table, t))) return rc;
    std::vector<float> tab(256);
    const Value& y = h->v[h->outv];
    for (int q = 0; q < 256; ++q) tab[q] = static_cast<float>(q - y.zero) * y.scale;
    if ((rc = upload(h, &h->head_table, tab))) return rc;
    CK(cudaMalloc(&h->ctc_terms, 256 * 256 * sizeof(float)));
    ctc_terms_kernel<<<256, 256, 0, h->stream>>>(h->head_table, h->ctc_terms);
    CK(cudaGetLastError());
    CK(cudaStreamSynchronize(h->stream));
  }
  const int ml = c->max_lines;
  const size_t frames = static_cast<size_t>(h->max_cols >> h->head_shift);
  h->max_pages = std::max(1, c->max_pages);
  CK(cudaStreamCreateWithFlags(&h->copy_stream, cudaStreamNonBlocking));
  for (auto& sl : h->slot) {
    CK(cudaEventCreateWithFlags(&sl.done, cudaEventDisableTiming));
    CK(cudaEventCreateWithFlags(&sl.unused, cudaEventDisableTiming));
    if ((rc = dev_alloc(h, &sl.d_pages, h->max_pages))) return rc;
  }
  h->d_pages = h->slot[0].d_pages;
  if ((rc = dev_alloc(h, &h->d_ext_pages, h->max_pages)) || (rc = dev_alloc(h, &h->d_lines, ml)) ||
      (rc = dev_alloc(h, &h->d_mask, h->max_cols / 8)) || (rc = dev_alloc(h, &h->d_frame0, ml)) ||
      (rc = dev_alloc(h, &h->d_length, ml)) || (rc = dev_alloc(h, &h->d_frame_id, frames)) ||
      (rc = dev_alloc(h, &h->d_frame_prob, frames)) || (rc = dev_alloc(h, &h->d_count, ml)) ||
      (rc = dev_alloc(h, &h->d_ids, frames)) || (rc = dev_alloc(h, &h->d_frames, frames)) ||
      (rc = dev_alloc(h, &h->d_probs, frames)) || (rc = dev_alloc(h, &h->d_err, 1)) ||
      (rc = dev_alloc(h, &h->d_claim, 2)) || (rc = dev_alloc(h, &h->d_wide_idx, ml)) ||
      (rc = dev_alloc(h, &h->d_order, ml)))
    return rc;
  CK(cudaMemset(h->d_claim, 0, 2 * sizeof(int)));
  if ((rc = host_alloc(h, &h->h_err, 1)) || (rc = host_alloc(h, &h->h_total, 1)) ||
      (rc = dev_alloc(h, &h->d_total, 1)))
    return rc;
  if (h->int8) {
    // the head's list: CTA b's part from b * region on, region = ceil(tiles / grid) x 128 entries
    h->nb_row_bytes = round16(h->v[h->outv].c);
    const size_t tiles = (frames + 127) / 128, entries = (tiles + h->sms - 1) / h->sms * h->sms * 128;
    if ((rc = dev_alloc(h, &h->d_nb_codes, entries * static_cast<size_t>(h->nb_row_bytes))) ||
        (rc = dev_alloc(h, &h->d_nb_frame, entries)) || (rc = dev_alloc(h, &h->d_nb_best, entries)) ||
        (rc = dev_alloc(h, &h->d_nb_count, 2 * static_cast<size_t>(h->sms))))
      return rc;
  }
  if (crop_smem_bytes(h, c->max_width) > 232448) return set_error(h, CREC_E_INVALID, "max_width: the crop kernel's shared memory");
  return CREC_OK;
}

int pages_common(crec_handle* h, const crec_page* pages, int n) {
  if (!h) return CREC_E_INVALID;
  if (h->broken) return set_error(h, CREC_E_STICKY, "the GPU is broken for this process");
  if (n < 0 || n > h->max_pages || (n > 0 && !pages)) return set_error(h, CREC_E_INVALID, "set_pages: page count");
  for (int i = 0; i < n; ++i)
    if (!pages[i].data || pages[i].width <= 0 || pages[i].height <= 0 || pages[i].stride < pages[i].width)
      return set_error(h, CREC_E_INVALID, "set_pages: page " + std::to_string(i));
  return CREC_OK;
}

}  // namespace

// ---------------------------------------------------------------- greedy CTC without allocating
//
// crec_ctc_greedy_noalloc's scratch: each frame's best class (int32) and probability (float), for
// at most kNoAllocFrames frames.  A file-scope device array: every GPU that loads this library
// holds these 4 MiB until the process exits, and every call on a device shares them.
constexpr size_t kNoAllocFrames = size_t{1} << 19;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocFrames * 8];

namespace {

constexpr int kNoAllocDevices = 64;
std::mutex g_noalloc_mutex;
void* g_noalloc_addr[kNoAllocDevices] = {};

// The scratch's device address on the current device, taken once per device (the host-side name
// g_noalloc_scratch is only a stand-in for it, not a device address).
cudaError_t noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kNoAllocDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_addr[dev]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_noalloc_addr[dev] = ptr;
  }
  *out = g_noalloc_addr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" {

int crec_width_bucket(int w) {
  for (int b = 32;;) {
    if (w <= b) return b;
    if (b >= 2048) return (w + 7) / 8 * 8;
    const int nb = (static_cast<int>(std::ceil(b * 1.3)) + 7) / 8 * 8;
    b = std::min(2048, nb);
  }
}

int crec_crop_region(const crec_box* box, const crec_crop_rule* r, double* region, int* width) {
  if (!box || !r || !region || !width) return CREC_E_INVALID;
  // carbon/src/lines.cpp:33-44: the same expressions, in the same order (built without contraction)
  const double h = box->y1 - box->y0;
  const double sy0 = box->y0 - r->pad_v * h, sy1 = box->y1 + r->pad_v * h;
  const double scale = r->height / (sy1 - sy0);
  const double w_src = (box->x1 - box->x0) + 2 * r->pad_h * h;
  const int w = std::max(r->width_step, static_cast<int>(std::ceil(w_src * scale / r->width_step - 1e-6)) * r->width_step);
  const double extra = (w / scale - w_src) / 2;
  region[0] = box->x0 - r->pad_h * h - extra;
  region[1] = sy0;
  region[2] = box->x1 + r->pad_h * h + extra;
  region[3] = sy1;
  *width = w;
  return CREC_OK;
}

int crec_open(const crec_config* config, crec_handle** out) {
  if (!config || !out) return CREC_E_INVALID;
  *out = nullptr;
  auto* h = new (std::nothrow) crec_handle();
  if (!h) return CREC_E_NOMEM;
  const int rc = open_impl(h, config);
  *out = h;  // the handle carries the error message even on failure; crec_close frees it
  return rc;
}

int crec_close(crec_handle* h) {
  if (!h) return CREC_OK;
  if (h->up_thread.joinable()) {
    {
      std::lock_guard<std::mutex> lk(h->up_m);
      h->up_stop = true;
    }
    h->up_cv.notify_all();
    h->up_thread.join();
  }
  h->stager.reset();
  cudaSetDevice(h->device);
  if (h->stream) cudaStreamSynchronize(h->stream);
  if (h->copy_stream) cudaStreamSynchronize(h->copy_stream);
  free_all(h);
  delete h;
  return CREC_OK;
}

const char* crec_last_error(const crec_handle* h) { return h ? h->error.c_str() : "no handle"; }
int crec_is_broken(const crec_handle* h) { return h && h->broken ? 1 : 0; }
void* crec_stream(crec_handle* h) { return h ? static_cast<void*>(h->stream) : nullptr; }

namespace {

// Whether host memory is page-locked (cudaHostAlloc'd or registered): the copy engine reads it as it is.
bool page_locked(const void* p) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeHost;
}

// The pages (only rows[i]'s runs where given) into a slot, queued on the copy stream once the
// recognize work that last read the slot is done; its `done` event follows them.  Page-locked
// pages are copied from where they are; pageable ones through the stager's pinned chunks.  Runs
// on the caller's thread (set_pages) or the uploader's (prefetch_pages); it touches the slot, the
// copy stream and the stager only (the handle's error message is the caller's to set).
int upload_slot(crec_handle* h, crec_handle::PageSlot& sl, const crec_page* pages, int n, const crec_row_runs* rows,
                std::string* msg) {
  auto fail = [&](int code, const std::string& m) {
    *msg = m;
    return code;
  };
  auto cuda = [&](cudaError_t e, const char* what) {
    if (e == cudaSuccess) return CREC_OK;
    cudaGetLastError();
    return fail(e == cudaErrorMemoryAllocation ? CREC_E_NOMEM : CREC_E_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  };
  int rc;
  size_t need = 0;
  for (int i = 0; i < n; ++i) need += (static_cast<size_t>(pages[i].height) * pages[i].width + 255) / 256 * 256;
  if (need > sl.cap) {
    const size_t limit = h->cfg.max_page_bytes > 0 ? static_cast<size_t>(h->cfg.max_page_bytes)
                                                   : static_cast<size_t>(h->max_pages) * 1700 * 2200;
    if (need > std::max(limit + static_cast<size_t>(n) * 256, sl.cap))
      return fail(CREC_E_RANGE, "set_pages: more page bytes than configured");
    // nothing queued may still read the old memory
    if ((rc = cuda(cudaStreamSynchronize(h->stream), "cudaStreamSynchronize")) ||
        (rc = cuda(cudaStreamSynchronize(h->copy_stream), "cudaStreamSynchronize")))
      return rc;
    cudaFree(sl.mem);
    sl.mem = nullptr;
    sl.cap = 0;
    if ((rc = cuda(cudaMalloc(&sl.mem, need), "cudaMalloc (pages)"))) return rc;
    sl.cap = need;
  }
  if (sl.recorded && (rc = cuda(cudaStreamWaitEvent(h->copy_stream, sl.unused, 0), "cudaStreamWaitEvent"))) return rc;
  sl.pages.resize(n);
  sl.views.assign(pages, pages + n);
  sl.bytes = 0;
  std::vector<RowPiece> staged;
  size_t at = 0;
  for (int i = 0; i < n; ++i) {
    const crec_page& pg = pages[i];
    uint8_t* d = sl.mem + at;
    sl.pages[i] = {d, pg.width, pg.height, static_cast<long long>(pg.width)};
    const bool locked = page_locked(pg.data);
    auto rows_of = [&](int y0, int y1) -> int {
      const uint8_t* src = pg.data + static_cast<long long>(y0) * pg.stride;
      uint8_t* dst = d + static_cast<size_t>(y0) * pg.width;
      sl.bytes += static_cast<long long>(y1 - y0) * pg.width;
      if (!locked) {
        staged.push_back({src, pg.stride, pg.width, y1 - y0, dst});
        return CREC_OK;
      }
      if (pg.stride == pg.width)  // contiguous rows: one copy
        return cuda(cudaMemcpyAsync(dst, src, static_cast<size_t>(y1 - y0) * pg.width, cudaMemcpyHostToDevice, h->copy_stream),
                    "cudaMemcpyAsync (pages)");
      return cuda(cudaMemcpy2DAsync(dst, pg.width, src, pg.stride, pg.width, y1 - y0, cudaMemcpyHostToDevice, h->copy_stream),
                  "cudaMemcpy2DAsync (pages)");
    };
    if (rows && rows[i].count > 0 && rows[i].runs) {
      for (int r = 0; r < rows[i].count; ++r) {
        const int y0 = std::max(0, rows[i].runs[2 * r]), y1 = std::min(pg.height, rows[i].runs[2 * r + 1]);
        if (y1 > y0 && (rc = rows_of(y0, y1))) return rc;
      }
    } else if ((rc = rows_of(0, pg.height))) {
      return rc;
    }
    at += (static_cast<size_t>(pg.height) * pg.width + 255) / 256 * 256;
  }
  if (!staged.empty()) {
    // 8 workers where the host has 16 CPUs or more (half of them on smaller hosts, for the caller's
    // own threads): measured on a 16-CPU B200 host with config 5's pageable pages, 4 workers with
    // plain memcpy sent 265-271 K lines/s, 8 with streaming stores 357 K; 12-14 no more, 16 fewer
    if (!h->stager) {
      const int hw = static_cast<int>(std::thread::hardware_concurrency());
      h->stager = std::make_unique<crec::Stager>(h->device, std::clamp(hw / 2, 2, kStagerWorkers));
    }
    if ((rc = cuda(h->stager->send(staged, h->copy_stream), "staged page upload"))) return rc;
  }
  if (n > 0 &&
      (rc = cuda(cudaMemcpyAsync(sl.d_pages, sl.pages.data(), sizeof(PageDesc) * n, cudaMemcpyHostToDevice, h->copy_stream),
                 "cudaMemcpyAsync (page descriptors)")))
    return rc;
  sl.bytes += static_cast<long long>(sizeof(PageDesc)) * n;
  return cuda(cudaEventRecord(sl.done, h->copy_stream), "cudaEventRecord");
}

// The uploader thread: one prefetch's upload at a time.  A failed prefetch leaves its slot not
// ready; the set_pages of those pages uploads them again and meets the error itself if it lasts.
void uploader(crec_handle* h) {
  cudaSetDevice(h->device);
  std::unique_lock<std::mutex> lk(h->up_m);
  for (;;) {
    h->up_cv.wait(lk, [&] { return h->up_stop || (h->up_busy && h->up_job.slot); });
    if (h->up_stop) return;
    crec_handle::UpJob job = std::move(h->up_job);
    h->up_job = {};
    lk.unlock();
    std::vector<crec_row_runs> rr(job.runs.size());
    for (size_t i = 0; i < rr.size(); ++i) rr[i] = {job.runs[i].data(), static_cast<int>(job.runs[i].size() / 2)};
    std::string msg;
    const int rc = upload_slot(h, *job.slot, job.pages.data(), static_cast<int>(job.pages.size()),
                               job.has_rows ? rr.data() : nullptr, &msg);
    lk.lock();
    if (rc) {
      job.slot->ready = false;
    } else {
      h->last_upload = job.slot->done;
      h->up_h2d += job.slot->bytes;
    }
    h->up_busy = false;
    h->up_cv.notify_all();
  }
}

// Until the uploader holds no prefetch (its copies queued, or its error met).
void wait_uploader(crec_handle* h) {
  std::unique_lock<std::mutex> lk(h->up_m);
  h->up_cv.wait(lk, [&] { return !h->up_busy; });
}

// The previous call's pages are the caller's again once its upload is done (the pages of a
// set_pages or prefetch_pages call stay alive until the next such call returns).
int release_previous(crec_handle* h) {
  wait_uploader(h);
  if (h->last_upload) CK(cudaEventSynchronize(h->last_upload));
  h->last_upload = nullptr;
  return CREC_OK;
}

bool same_pages(const std::vector<crec_page>& a, const crec_page* b, int n) {
  if (static_cast<int>(a.size()) != n) return false;
  for (int i = 0; i < n; ++i)
    if (a[i].data != b[i].data || a[i].width != b[i].width || a[i].height != b[i].height || a[i].stride != b[i].stride)
      return false;
  return true;
}

}  // namespace

int crec_set_pages(crec_handle* h, const crec_page* pages, int n, const crec_row_runs* rows) {
  int rc = pages_common(h, pages, n);
  if (rc) return rc;
  CK(cudaSetDevice(h->device));
  h->st_h2d = 0;
  h->st_d2h = 0;
  h->st_launches = 0;
  h->st_runs = 0;
  if ((rc = release_previous(h))) return rc;  // a taken prefetch's upload too: done by now when it ran beside a group
  crec_handle::PageSlot& next = h->slot[1 - h->cur];
  const bool taken = next.ready && same_pages(next.views, pages, n);
  if (!taken) {
    std::string msg;
    if ((rc = upload_slot(h, next, pages, n, rows, &msg))) return set_error(h, rc, msg);
    h->last_upload = next.done;
    h->tot_h2d += next.bytes;
  }
  h->st_h2d = next.bytes;
  next.ready = false;
  // the slot left behind is free once the recognize work queued so far is done
  crec_handle::PageSlot& old = h->slot[h->cur];
  CK(cudaEventRecord(old.unused, h->stream));
  old.recorded = true;
  h->cur = 1 - h->cur;
  h->pages = next.pages;
  h->d_pages = next.d_pages;
  CK(cudaStreamWaitEvent(h->stream, next.done, 0));  // the recognize stream waits for the upload alone
  return CREC_OK;
}

int crec_prefetch_pages(crec_handle* h, const crec_page* pages, int n, const crec_row_runs* rows) {
  int rc = pages_common(h, pages, n);
  if (rc) return rc;
  CK(cudaSetDevice(h->device));
  if ((rc = release_previous(h))) return rc;
  crec_handle::PageSlot& next = h->slot[1 - h->cur];
  crec_handle::UpJob job;
  job.slot = &next;
  job.pages.assign(pages, pages + n);
  job.has_rows = rows != nullptr;
  if (rows) {
    job.runs.resize(n);
    for (int i = 0; i < n; ++i)
      if (rows[i].count > 0 && rows[i].runs) job.runs[i].assign(rows[i].runs, rows[i].runs + 2 * rows[i].count);
  }
  next.views = job.pages;  // what set_pages compares; the upload writes the same
  next.ready = true;
  if (!h->up_thread.joinable()) h->up_thread = std::thread(uploader, h);
  {
    std::lock_guard<std::mutex> lk(h->up_m);
    h->up_job = std::move(job);
    h->up_busy = true;
  }
  h->up_cv.notify_all();
  return CREC_OK;
}

int crec_set_pages_device(crec_handle* h, const crec_page* pages, int n) {
  int rc = pages_common(h, pages, n);
  if (rc) return rc;
  CK(cudaSetDevice(h->device));
  h->pages.resize(n);
  for (int i = 0; i < n; ++i) h->pages[i] = {pages[i].data, pages[i].width, pages[i].height, static_cast<long long>(pages[i].stride)};
  if (n > 0) CK(cudaMemcpyAsync(h->d_ext_pages, h->pages.data(), sizeof(PageDesc) * n, cudaMemcpyHostToDevice, h->stream));
  CK(cudaStreamSynchronize(h->stream));
  h->d_pages = h->d_ext_pages;
  return CREC_OK;
}

int crec_recognize(crec_handle* h, const int32_t* page_of, const crec_box* boxes, int n, int bw, crec_lines* out) {
  if (!h) return CREC_E_INVALID;
  if (h->broken) return set_error(h, CREC_E_STICKY, "the GPU is broken for this process");
  if (n < 0 || n > h->cfg.max_lines) return set_error(h, CREC_E_RANGE, "recognize: more lines than max_lines");
  if (bw <= 0 || bw > h->cfg.max_width || bw % h->cfg.crop.width_step || bw % (1 << h->max_shift))
    return set_error(h, CREC_E_INVALID, "recognize: bucket width " + std::to_string(bw));
  if (!out || (n > 0 && (!page_of || !boxes || !out->counts || !out->lengths || !out->offsets || !out->ids ||
                          !out->frames || !out->probs)))
    return set_error(h, CREC_E_INVALID, "recognize: null arrays");
  out->total = 0;
  if (n == 0) return CREC_OK;
  CK(cudaSetDevice(h->device));
  std::vector<int> bws(n, bw);
  Source src;
  src.page_of = page_of;
  src.boxes = boxes;
  return recognize_all(h, src, bws.data(), n, out);
}

int crec_recognize_lines(crec_handle* h, const int32_t* page_of, const crec_box* boxes, const int32_t* bw, int n,
                         crec_lines* out) {
  if (!h) return CREC_E_INVALID;
  if (h->broken) return set_error(h, CREC_E_STICKY, "the GPU is broken for this process");
  if (n < 0 || !out || (n > 0 && (!page_of || !boxes || !out->counts || !out->lengths || !out->offsets ||
                                   !out->ids || !out->frames || !out->probs)))
    return set_error(h, CREC_E_INVALID, "recognize_lines: arguments");
  out->total = 0;
  if (n == 0) return CREC_OK;
  CK(cudaSetDevice(h->device));
  std::vector<int> bws(n);
  // a bucket width is a multiple of the width step and of the network's horizontal stride (a
  // power of two): with a power-of-two step both are one mask, without a division a line
  const int step = h->cfg.crop.width_step;
  const bool pow2 = step > 0 && (step & (step - 1)) == 0;
  const int mask = ((1 << h->max_shift) - 1) | (pow2 ? step - 1 : 0);
  for (int i = 0; i < n; ++i) {
    if (bw) {
      bws[i] = bw[i];
    } else {
      double reg[4];
      int w = 0;
      crec_crop_region(&boxes[i], &h->cfg.crop, reg, &w);
      bws[i] = crec_width_bucket(w);
    }
    if (bws[i] <= 0 || bws[i] > h->cfg.max_width || (bws[i] & mask) || (!pow2 && bws[i] % step))
      return set_error(h, CREC_E_INVALID, "recognize_lines: line " + std::to_string(i) + " bucket width " + std::to_string(bws[i]));
  }
  Source src;
  src.page_of = page_of;
  src.boxes = boxes;
  return recognize_all(h, src, bws.data(), n, out);
}

int crec_recognize_crops(crec_handle* h, const uint8_t* crops, int pitch, const int32_t* widths, const int32_t* bw,
                         int n, crec_lines* out) {
  if (!h) return CREC_E_INVALID;
  if (h->broken) return set_error(h, CREC_E_STICKY, "the GPU is broken for this process");
  if (n < 0 || !out || (n > 0 && (!crops || !widths || !bw)) || pitch <= 0 || pitch > h->cfg.max_width)
    return set_error(h, CREC_E_INVALID, "recognize_crops: arguments");
  out->total = 0;
  if (n == 0) return CREC_OK;
  CK(cudaSetDevice(h->device));
  for (int i = 0; i < n; ++i)
    if (bw[i] <= 0 || bw[i] > pitch || bw[i] % h->cfg.crop.width_step || bw[i] % (1 << h->max_shift))
      return set_error(h, CREC_E_INVALID, "recognize_crops: line " + std::to_string(i) + " bucket width " + std::to_string(bw[i]));
  if (!h->d_crops_in) CK(cudaMalloc(&h->d_crops_in, static_cast<size_t>(h->cfg.max_lines) * h->height * h->cfg.max_width));
  std::vector<int> bws(bw, bw + n);
  Source src;
  src.crops = crops;
  src.pitch = pitch;
  src.widths = widths;
  return recognize_all(h, src, bws.data(), n, out);
}

int crec_debug_crops(crec_handle* h, uint8_t* out, int pitch) {
  if (!h || pitch <= 0) return CREC_E_INVALID;
  CK(cudaSetDevice(h->device));
  if (!out) {  // arm: the runs from now on keep their finished crops
    cudaFree(h->d_crops);
    h->d_crops = nullptr;
    CK(cudaMalloc(&h->d_crops, static_cast<size_t>(h->cfg.max_lines) * h->height * pitch));
    CK(cudaMemset(h->d_crops, 0, static_cast<size_t>(h->cfg.max_lines) * h->height * pitch));
    h->crops_pitch = pitch;
    return CREC_OK;
  }
  if (!h->d_crops || h->crops_pitch != pitch) return set_error(h, CREC_E_INVALID, "debug crops not armed at this pitch");
  CK(cudaMemcpy(out, h->d_crops, static_cast<size_t>(h->last_n) * h->height * pitch, cudaMemcpyDeviceToHost));
  return CREC_OK;
}

int crec_ctc_greedy(const float* logits, int n, int classes, int frames, const int32_t* lengths, crec_lines* out,
                    void* stream, char* error, size_t error_size) {
  auto fail = [&](int code, const std::string& msg) {
    if (error && error_size) {
      std::snprintf(error, error_size, "%s", msg.c_str());
    }
    return code;
  };
  if (n < 0 || classes <= 0 || frames < 0 || (n > 0 && (!logits || !lengths || !out)))
    return fail(CREC_E_INVALID, "ctc_greedy: arguments");
  if (!out) return fail(CREC_E_INVALID, "ctc_greedy: no output");
  out->total = 0;
  if (n == 0 || frames == 0) {
    for (int i = 0; i < n; ++i) out->counts[i] = out->lengths[i] = out->offsets[i] = 0;
    return CREC_OK;
  }
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t cells = static_cast<size_t>(n) * frames;
  // per-call scratch (stream-ordered): lengths, each frame's best class and probability, the slots, counts
  int32_t *d_len = nullptr, *d_arg = nullptr, *d_ids = nullptr, *d_starts = nullptr, *d_count = nullptr;
  float *d_prob = nullptr, *d_probs = nullptr;
  auto release = [&]() {
    cudaFreeAsync(d_len, s);
    cudaFreeAsync(d_arg, s);
    cudaFreeAsync(d_ids, s);
    cudaFreeAsync(d_starts, s);
    cudaFreeAsync(d_count, s);
    cudaFreeAsync(d_prob, s);
    cudaFreeAsync(d_probs, s);
  };
  cudaError_t e = cudaSuccess;
  if ((e = cudaMallocAsync(&d_len, sizeof(int32_t) * n, s)) != cudaSuccess ||
      (e = cudaMallocAsync(&d_arg, sizeof(int32_t) * cells, s)) != cudaSuccess ||
      (e = cudaMallocAsync(&d_ids, sizeof(int32_t) * cells, s)) != cudaSuccess ||
      (e = cudaMallocAsync(&d_starts, sizeof(int32_t) * cells, s)) != cudaSuccess ||
      (e = cudaMallocAsync(&d_count, sizeof(int32_t) * n, s)) != cudaSuccess ||
      (e = cudaMallocAsync(&d_prob, sizeof(float) * cells, s)) != cudaSuccess ||
      (e = cudaMallocAsync(&d_probs, sizeof(float) * cells, s)) != cudaSuccess) {
    release();
    return fail(e == cudaErrorMemoryAllocation ? CREC_E_NOMEM : CREC_E_CUDA,
                std::string("ctc_greedy: ") + cudaGetErrorString(e));
  }
  std::vector<int32_t> count(n), ids(cells), starts(cells);
  std::vector<float> probs(cells);
  e = cudaMemcpyAsync(d_len, lengths, sizeof(int32_t) * n, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) {
    ctc_argmax_kernel<<<n, 256, 0, s>>>(logits, classes, frames, d_len, d_arg, d_prob);
    ctc_collapse_lines_kernel<<<(n + 127) / 128, 128, 0, s>>>(n, frames, d_len, d_arg, d_prob, d_ids, d_starts,
                                                               d_probs, d_count);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaMemcpyAsync(count.data(), d_count, sizeof(int32_t) * n, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(ids.data(), d_ids, sizeof(int32_t) * cells, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(starts.data(), d_starts, sizeof(int32_t) * cells, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(probs.data(), d_probs, sizeof(float) * cells, cudaMemcpyDeviceToHost, s);
  release();
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return fail(CREC_E_CUDA, std::string("ctc_greedy: ") + cudaGetErrorString(e));
  for (int i = 0; i < n; ++i) {
    const int k = count[i];
    out->counts[i] = k;
    out->lengths[i] = std::min(std::max(lengths[i], 0), frames);
    out->offsets[i] = static_cast<int32_t>(out->total);
    if (out->total + k > out->capacity) return fail(CREC_E_RANGE, "ctc_greedy: crec_lines capacity too small");
    const size_t b = static_cast<size_t>(i) * frames;
    std::memcpy(out->ids + out->total, ids.data() + b, sizeof(int32_t) * k);
    std::memcpy(out->frames + out->total, starts.data() + b, sizeof(int32_t) * k);
    std::memcpy(out->probs + out->total, probs.data() + b, sizeof(float) * k);
    out->total += k;
  }
  return CREC_OK;
}

int crec_ctc_greedy_noalloc(const float* logits, int n, int classes, int frames, const int32_t* lengths,
                            int32_t* counts, int32_t* ids, int32_t* starts, float* probs, void* stream, char* error,
                            size_t error_size) {
  auto fail = [&](int code, const char* msg) {
    if (error && error_size) std::snprintf(error, error_size, "%s", msg);
    return code;
  };
  // every line gets a count (and reads its length), so those two are needed whenever there are
  // lines; the logits and the character arrays only when there are frames to read
  if (n < 0 || classes <= 0 || frames < 0 || (n > 0 && (!lengths || !counts)) ||
      (n > 0 && frames > 0 && (!logits || !ids || !starts || !probs)))
    return fail(CREC_E_INVALID, "ctc_greedy_noalloc: arguments");
  const size_t cells = static_cast<size_t>(n) * static_cast<size_t>(frames);
  if (cells > kNoAllocFrames) {
    char msg[160];
    std::snprintf(msg, sizeof msg, "ctc_greedy_noalloc: n x frames = %zu frames, more than its scratch's %zu",
                  cells, kNoAllocFrames);
    return fail(CREC_E_RANGE, msg);
  }
  if (n == 0) return CREC_OK;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (frames == 0) {  // no frames: every line has no characters; no kernel, no scratch
    e = cudaMemsetAsync(counts, 0, sizeof(int32_t) * static_cast<size_t>(n), s);
    return e == cudaSuccess ? CREC_OK : fail(CREC_E_CUDA, cudaGetErrorString(e));
  }
  void* scratch = nullptr;
  e = noalloc_scratch(&scratch);
  if (e != cudaSuccess) return fail(CREC_E_CUDA, cudaGetErrorString(e));
  int32_t* arg = static_cast<int32_t*>(scratch);
  float* prob = reinterpret_cast<float*>(static_cast<uint8_t*>(scratch) + kNoAllocFrames * 4);
  // nothing in the scratch needs to start at zero: the argmax writes every frame the collapse reads
  ctc_argmax_kernel<<<n, 256, 0, s>>>(logits, classes, frames, lengths, arg, prob);
  ctc_collapse_lines_kernel<<<(n + 127) / 128, 128, 0, s>>>(n, frames, lengths, arg, prob, ids, starts, probs, counts);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(CREC_E_CUDA, cudaGetErrorString(e));
  return CREC_OK;
}

int crec_debug_inject(crec_handle* h, int what) {
  if (!h) return CREC_E_INVALID;
  if (what == CREC_INJECT_TIMEOUT) h->inject_timeout = true;
  else if (what == CREC_INJECT_STICKY) h->inject_sticky = true;
  else return set_error(h, CREC_E_INVALID, "debug_inject: what");
  return CREC_OK;
}

int crec_candidates(crec_handle* h, const int32_t* rows, int n, int topk, int32_t* k_out, int32_t* frames, int32_t* ids,
                    float* logp, float* blank, int64_t capacity) {
  if (!h) return CREC_E_INVALID;
  if (h->broken) return set_error(h, CREC_E_STICKY, "the GPU is broken for this process");
  if (n < 0 || !k_out || (n > 0 && (!rows || !frames || !blank)) || (n > 0 && topk > 0 && (!ids || !logp)))
    return set_error(h, CREC_E_INVALID, "candidates: arguments");
  const Layer& head = h->l.back();
  const Value& x = h->v[head.in];
  const Value& xp = h->v[x.phys];
  const int classes = h->v[head.out].c;
  // as the reference's GPU device clamps it (carbon/src/cuda/pipeline_cuda.cpp:501)
  topk = std::clamp(topk, 0, std::min(classes - 1, 16));
  *k_out = topk;
  std::vector<int32_t> cols;
  for (int j = 0; j < n; ++j) {
    const int r = rows[j] - h->last_a;
    if (r < 0 || r >= h->last_n)
      return set_error(h, CREC_E_RANGE, "candidates: line " + std::to_string(rows[j]) +
                                            " is not in the last run of the last recognize call");
    frames[j] = h->last_len[r];
    for (int t = 0; t < h->last_len[r]; ++t) cols.push_back(h->last_frame0[r] + t);
  }
  const size_t total = cols.size();
  if (static_cast<int64_t>(total) > capacity) return set_error(h, CREC_E_RANGE, "candidates: capacity too small");
  if (total == 0) return CREC_OK;
  CK(cudaSetDevice(h->device));
  cudaStream_t s = h->stream;
  const size_t cells = total * std::max(topk, 1);
  size_t cap_f = h->cap_cand_frames, cap_f2 = 3 * cap_f, cap_c = h->cap_cand_cells, cap_c2 = cap_c;
  int rc;
  if ((rc = grow_device(h, &h->d_cand_cols, &cap_f, total)) || (rc = grow_device(h, &h->d_cand_fr, &cap_f2, 3 * total)) ||
      (rc = grow_device(h, &h->d_cand_ids, &cap_c, cells)) || (rc = grow_device(h, &h->d_cand_vals, &cap_c2, cells)))
    return rc;
  h->cap_cand_frames = std::min(cap_f, cap_f2 / 3);
  h->cap_cand_cells = std::min(cap_c, cap_c2);
  CK(cudaMemcpyAsync(h->d_cand_cols, cols.data(), sizeof(int32_t) * total, cudaMemcpyHostToDevice, s));
  CandParams p{};
  p.x = xp.base + static_cast<long long>(xp.ph) * xp.pitch;
  p.cp = x.cp;
  p.k = x.cp;
  p.classes = classes;
  p.topk = topk;
  p.w8 = head.dw8;
  p.wf = head.dwf;
  p.colsum = head.colsum;
  p.scale = head.scale;
  p.bias = head.dbias;
  p.in_zero = x.zero;
  p.out_zero = h->v[head.out].zero;
  p.out_inv_scale = h->int8 ? 1.0f / h->v[head.out].scale : 1.0f;
  p.table = h->head_table;
  p.cols = h->d_cand_cols;
  p.frames = static_cast<int>(total);
  p.ids = h->d_cand_ids;
  p.vals = h->d_cand_vals;
  p.best = h->d_cand_fr;
  p.sum = h->d_cand_fr + total;
  p.blank = h->d_cand_fr + 2 * total;
  const int smem = classes * 4 + static_cast<int>(round16(x.cp * h->eb));
  auto* k = h->int8 ? candidates_kernel<true> : candidates_kernel<false>;
  CK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  k<<<static_cast<unsigned>(total), kCandThreads, smem, s>>>(p);
  CK(cudaGetLastError());
  std::vector<float> fr(3 * total), vals(cells);
  if (topk > 0) {
    CK(cudaMemcpyAsync(ids, h->d_cand_ids, sizeof(int32_t) * total * topk, cudaMemcpyDeviceToHost, s));
    CK(cudaMemcpyAsync(vals.data(), h->d_cand_vals, sizeof(float) * total * topk, cudaMemcpyDeviceToHost, s));
  }
  CK(cudaMemcpyAsync(fr.data(), h->d_cand_fr, sizeof(float) * 3 * total, cudaMemcpyDeviceToHost, s));
  CK(cudaStreamSynchronize(s));
  // carbon/src/cpu/kernels.cpp:658-664: each frame's offset best + ln(sum), in float with the C
  // library's logf, as the CPU reference takes it
  for (size_t f = 0; f < total; ++f) {
    const float off = fr[f] + std::log(fr[total + f]);
    for (int q = 0; q < topk; ++q) logp[f * topk + q] = vals[f * topk + q] - off;
    blank[f] = fr[2 * total + f] - off;
  }
  return CREC_OK;
}

int crec_last_stats(const crec_handle* h, crec_stats* out) {
  if (!h || !out) return CREC_E_INVALID;
  out->runs = h->st_runs;
  out->launches = h->st_launches;
  out->h2d_bytes = h->st_h2d;
  out->d2h_bytes = h->st_d2h;
  {
    std::lock_guard<std::mutex> lk(const_cast<crec_handle*>(h)->up_m);
    out->h2d_total = h->tot_h2d + h->up_h2d;
  }
  out->d2h_total = h->tot_d2h;
  out->wide_lines = h->st_wide;
  return CREC_OK;
}

int crec_profile(crec_handle* h, int enable, crec_profile_entry* out, int capacity) {
  if (!h) return CREC_E_INVALID;
  static const char* names[5] = {"crop_stem", "conv_gemm_tcgen05", "depthwise", "head_ctc_tcgen05", "collapse"};
  int n = 0;
  if (out) {
    for (int k = 0; k < 5 && n < capacity; ++k, ++n) {
      out[n].kernel = names[k];
      out[n].launches = h->prof_count[k];
      out[n].ms = h->prof_ms[k];
      out[n].ops = h->prof_ops[k];
    }
  }
  if (enable >= 0) {  // (re)start: clear the totals
    h->profile = enable != 0;
    h->lprof_ms.assign(h->l.size() + 1, 0.0);
    h->lprof_ops.assign(h->l.size() + 1, 0.0);
    h->lprof_count.assign(h->l.size() + 1, 0);
    for (int k = 0; k < 8; ++k) {
      h->prof_ms[k] = 0;
      h->prof_ops[k] = 0;
      h->prof_count[k] = 0;
    }
  }
  return n;
}

int crec_profile_layers(crec_handle* h, crec_profile_entry* out, int capacity) {
  if (!h || (!out && capacity > 0)) return CREC_E_INVALID;
  const size_t nl = h->l.size();
  int n = 0;
  for (size_t li = 0; li <= nl && n < capacity; ++li, ++n) {
    const char* name = "collapse";
    if (li < nl) {
      const Layer& l = h->l[li];
      name = li == 0                   ? "crop_stem"
             : li + 1 == nl            ? "head_ctc_tcgen05"
             : l.kind == kKindDw       ? "depthwise"
             : l.kind == kKindResize   ? "resize (read in place)"
                                       : "conv_gemm_tcgen05";
    }
    out[n].kernel = name;
    out[n].launches = li < h->lprof_count.size() ? h->lprof_count[li] : 0;
    out[n].ms = li < h->lprof_ms.size() ? h->lprof_ms[li] : 0.0;
    out[n].ops = li < h->lprof_ops.size() ? h->lprof_ops[li] : 0.0;
  }
  return n;
}

int crec_debug_logits(crec_handle* h, float* out, int64_t capacity) {
  if (!h) return CREC_E_INVALID;
  CK(cudaSetDevice(h->device));
  const int classes = h->v[h->outv].c;
  if (!out) {  // arm: the runs from now on write their logits
    if (!h->d_logits) CK(cudaMalloc(&h->d_logits, static_cast<size_t>(h->max_cols >> h->head_shift) * classes * sizeof(float)));
    return CREC_OK;
  }
  if (!h->d_logits) return set_error(h, CREC_E_INVALID, "debug logits not armed");
  CK(cudaStreamSynchronize(h->stream));
  size_t need = 0;
  for (int i = 0; i < h->last_n; ++i) need += static_cast<size_t>(h->last_bw[i] >> h->head_shift) * classes;
  if (static_cast<int64_t>(need) > capacity) return set_error(h, CREC_E_RANGE, "debug_logits: capacity");
  float* o = out;
  for (int i = 0; i < h->last_n; ++i) {  // line i: [classes][frames], as the reference's output
    const long long f0 = h->last_seg[i] >> h->head_shift, t = h->last_bw[i] >> h->head_shift;
    std::vector<float> buf(static_cast<size_t>(t) * classes);
    CK(cudaMemcpy(buf.data(), h->d_logits + f0 * classes, buf.size() * sizeof(float), cudaMemcpyDeviceToHost));
    for (long long f = 0; f < t; ++f)
      for (int c = 0; c < classes; ++c) o[static_cast<size_t>(c) * t + f] = buf[static_cast<size_t>(f) * classes + c];
    o += buf.size();
  }
  return CREC_OK;
}

int crec_debug_value(crec_handle* h, int value, void* out, int64_t capacity) {
  if (!h || !out || value < 0 || value >= static_cast<int>(h->v.size())) return CREC_E_INVALID;
  const Value& v = h->v[value];
  if (v.h < 0) return set_error(h, CREC_E_INVALID, "value not computed");
  const Value& pv = h->v[v.phys];
  if (!pv.real) return set_error(h, CREC_E_INVALID, "value not kept in memory (the input or the head's output)");
  CK(cudaSetDevice(h->device));
  CK(cudaStreamSynchronize(h->stream));
  const size_t px = static_cast<size_t>(v.c) * h->eb;
  size_t need = 0;
  for (int i = 0; i < h->last_n; ++i) need += static_cast<size_t>(v.h) * (h->last_bw[i] >> v.shift) * px;
  if (static_cast<int64_t>(need) > capacity) return set_error(h, CREC_E_RANGE, "debug_value: capacity");
  std::vector<uint8_t> row(static_cast<size_t>(pv.pitch));
  uint8_t* o = static_cast<uint8_t*>(out);
  for (int i = 0; i < h->last_n; ++i) {
    const long long c0 = h->last_seg[i] >> v.shift, w = h->last_bw[i] >> v.shift;
    for (int y = 0; y < v.h; ++y) {
      CK(cudaMemcpy(row.data(), pv.base + static_cast<long long>(y + pv.ph) * pv.pitch, row.size(), cudaMemcpyDeviceToHost));
      for (long long x = 0; x < w; ++x) {
        const long long pcol = x + c0;  // logical column; the physical one for an upsampling read in place
        const long long src = (pcol >> v.extra) * pv.cp * h->eb;
        std::memcpy(o, row.data() + src, px);
        o += px;
      }
    }
  }
  return CREC_OK;
}

}  // extern "C"

namespace {

// Opens `h` as a layer-only device (no crop, no head): the blob's one dense convolution between
// its input value (h_in rows) and output value, each input line bw columns wide, n of them laid
// out as a run is; the layer set up exactly as in a recognizer (setup_layer, the same tensors).
// A bare handle for one layer of a blob on `device` (the sweeps): the device, its tensor-map
// encoder, a stream, the blob read.
int open_device(crec_handle* h, int device, int precision, const void* model, size_t model_bytes) {
  h->int8 = precision == CREC_INT8;
  h->eb = h->int8 ? 1 : 2;
  h->device = device;
  CK(cudaSetDevice(device));
  cudaDeviceProp prop{};
  CK(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10) return set_error(h, CREC_E_INVALID, "this build runs on sm_100 (B200)");
  h->sms = prop.multiProcessorCount;
  cudaDriverEntryPointQueryResult q{};
  void* fn = nullptr;
  CK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
  if (!fn || q != cudaDriverEntryPointSuccess) return set_error(h, CREC_E_CUDA, "cuTensorMapEncodeTiled is not available");
  h->encode = reinterpret_cast<EncodeTiled>(fn);
  CK(cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking));
  return read_model(h, static_cast<const uint8_t*>(model), model_bytes);
}

int open_layer(crec_handle* h, int device, int precision, const void* model, size_t model_bytes, int n, int h_in,
               int bw, long long* cols_out) {
  int rc = open_device(h, device, precision, model, model_bytes);
  if (rc) return rc;
  if (h->l.size() != 1 || h->l[0].kind != kKindConv || h->l[0].residual >= 0)
    return set_error(h, CREC_E_MODEL, "a blob of one dense convolution");
  const Layer conv = h->l[0];
  Value& x = h->v[conv.in];
  Value& y = h->v[conv.out];
  const int s = log2i(conv.sw);
  if (s < 0 || conv.kh > 3 || x.c % 16 || y.c % 16) return set_error(h, CREC_E_MODEL, "a convolution this sweep does not run");
  x.h = h_in;
  x.shift = 0;
  x.phys = conv.in;
  x.real = true;
  x.cp = x.c;
  y.h = (h_in + conv.pt + conv.pb - conv.kh) / conv.sh + 1;
  y.shift = s;
  y.phys = conv.out;
  y.real = true;
  y.cp = y.c;
  if (y.h <= 0 || bw % (8 << s)) return set_error(h, CREC_E_INVALID, "layer sweep: shape");
  h->max_shift = s;
  h->head_shift = s;
  h->gap = static_cast<int>(round_up(std::max({1, conv.pl, conv.pr}), std::max(8, 1 << s)));
  Layer stub{};
  stub.kind = kKindResize;
  h->l = {stub, conv, stub};  // setup_layer's view: neither the first layer (the stem) nor the last (the head)
  const long long cols = round_up(static_cast<long long>(n) * (bw + h->gap) + h->gap, 128LL << s);
  h->max_cols = cols;
  if ((rc = setup_layer(h, 1)) || (rc = alloc_values(h))) return rc;
  if ((rc = dev_alloc(h, &h->d_mask, static_cast<size_t>(cols / 8))) || (rc = dev_alloc(h, &h->d_err, 1))) return rc;
  std::vector<uint8_t> mask(static_cast<size_t>(cols / 8), 0);
  for (int i = 0; i < n; ++i) std::memset(mask.data() + (h->gap + static_cast<long long>(i) * (bw + h->gap)) / 8, 1, bw / 8);
  CK(cudaMemcpy(h->d_mask, mask.data(), mask.size(), cudaMemcpyHostToDevice));
  CK(cudaMemset(h->d_err, 0, sizeof(int)));
  *cols_out = cols;
  return CREC_OK;
}

// A handle for a blob of one 1x1 convolution run as the recognizer's head over `frames` frames of
// one row: the frames at input columns [gap, gap + frames), every column the head computes
// masked in (the mask's 8-column groups).
int open_head(crec_handle* h, int device, int precision, const void* model, size_t model_bytes, int frames,
              long long* cols_out) {
  int rc = open_device(h, device, precision, model, model_bytes);
  if (rc) return rc;
  if (h->l.size() != 1 || h->l[0].kind != kKindConv || h->l[0].residual >= 0 || h->l[0].kh != 1 || h->l[0].kw != 1 ||
      h->l[0].sh != 1 || h->l[0].sw != 1 || h->l[0].pl || h->l[0].pr || h->l[0].pt || h->l[0].pb)
    return set_error(h, CREC_E_MODEL, "a blob of one 1x1 convolution");
  const Layer head = h->l[0];
  Value& x = h->v[head.in];
  Value& y = h->v[head.out];
  if ((x.c * h->eb) % 16) return set_error(h, CREC_E_MODEL, "a head input of whole 16-byte channel groups");
  if (h->int8 && !y.u8) return set_error(h, CREC_E_MODEL, "the INT8 head's output must be quantized (Q/DQ)");
  x.h = 1;
  x.shift = 0;
  x.phys = head.in;
  x.real = true;
  x.cp = x.c;
  y.h = 1;
  y.shift = 0;
  y.phys = head.out;
  y.real = false;
  h->max_shift = 0;
  h->head_shift = 0;
  h->gap = 8;
  Layer stub{};
  stub.kind = kKindResize;
  h->l = {stub, head};  // setup_layer's view: the last layer (the head), not the first (the stem)
  const long long cols = round_up(static_cast<long long>(h->gap) + frames, 128LL);
  h->max_cols = cols;
  if ((rc = setup_layer(h, 1)) || (rc = alloc_values(h))) return rc;
  const size_t ncols = static_cast<size_t>(cols);
  if ((rc = dev_alloc(h, &h->d_mask, ncols / 8)) || (rc = dev_alloc(h, &h->d_err, 1)) ||
      (rc = dev_alloc(h, &h->d_frame_id, ncols)) || (rc = dev_alloc(h, &h->d_frame_prob, ncols)) ||
      (rc = dev_alloc(h, &h->d_logits, ncols * static_cast<size_t>(y.c))))
    return rc;
  if (h->int8) {
    std::vector<float> tab(256);
    for (int q = 0; q < 256; ++q) tab[q] = static_cast<float>(q - y.zero) * y.scale;
    if ((rc = upload(h, &h->head_table, tab))) return rc;
    CK(cudaMalloc(&h->ctc_terms, 256 * 256 * sizeof(float)));
    ctc_terms_kernel<<<256, 256, 0, h->stream>>>(h->head_table, h->ctc_terms);
    CK(cudaGetLastError());
    h->nb_row_bytes = round16(y.c);
    const size_t tiles = (ncols + 127) / 128, entries = (tiles + h->sms - 1) / h->sms * h->sms * 128;
    if ((rc = dev_alloc(h, &h->d_nb_codes, entries * static_cast<size_t>(h->nb_row_bytes))) ||
        (rc = dev_alloc(h, &h->d_nb_frame, entries)) || (rc = dev_alloc(h, &h->d_nb_best, entries)) ||
        (rc = dev_alloc(h, &h->d_nb_count, 2 * static_cast<size_t>(h->sms))))
      return rc;
  }
  std::vector<uint8_t> mask(ncols / 8, 0);
  std::memset(mask.data() + h->gap / 8, 1, static_cast<size_t>((frames + 7) / 8));
  CK(cudaMemcpy(h->d_mask, mask.data(), mask.size(), cudaMemcpyHostToDevice));
  CK(cudaMemset(h->d_err, 0, sizeof(int)));
  CK(cudaStreamSynchronize(h->stream));
  *cols_out = cols;
  return CREC_OK;
}

}  // namespace

int crec_ctc_head_blob(const void* file, size_t bytes, void* blob, size_t capacity, size_t* blob_bytes, char* error,
                       size_t error_size) {
  auto fail = [&](const std::string& m) {
    if (error && error_size) std::snprintf(error, error_size, "%s", m.c_str());
    return CREC_E_MODEL;
  };
  if (!file || !blob_bytes) return CREC_E_INVALID;
  // carbon/src/lines.cpp:372-398 (load_ctc_head): "CTCHEAD1", int32 classes, int32 k, the weight
  // [classes][k] in float16, the bias [classes] in float32, little-endian, nothing after
  const uint8_t* b = static_cast<const uint8_t*>(file);
  constexpr size_t kHeader = 16;
  if (bytes < kHeader || std::memcmp(b, "CTCHEAD1", 8) != 0)
    return fail("not a CTC head (the export writes <model>.head.bin)");
  int32_t dims[2];
  std::memcpy(dims, b + 8, sizeof dims);
  const int classes = dims[0], k = dims[1];
  const size_t cells = static_cast<size_t>(std::max(classes, 0)) * static_cast<size_t>(std::max(k, 0));
  const size_t want = kHeader + cells * 2 + static_cast<size_t>(std::max(classes, 0)) * 4;
  if (classes <= 0 || k <= 0 || bytes != want)
    return fail("a head of " + std::to_string(classes) + " classes by " + std::to_string(k) + " takes " +
                std::to_string(want) + " bytes, the file has " + std::to_string(bytes));
  // a CRECMDL1 float blob of the one 1x1 convolution, k channels to `classes` (as netdef writes it)
  const size_t need = 8 + 8 * 4 + 2 * 24 + 20 * 4 + cells * 4 + static_cast<size_t>(classes) * 4;
  *blob_bytes = need;
  if (!blob || capacity < need) return CREC_E_RANGE;
  uint8_t* o = static_cast<uint8_t*>(blob);
  auto put = [&](const void* v, size_t n) {
    std::memcpy(o, v, n);
    o += n;
  };
  auto u32 = [&](uint32_t v) { put(&v, 4); };
  put("CRECMDL1", 8);
  for (uint32_t v : {1u, 1u, 2u, 1u, 0u, 1u, 1u, 0u}) u32(v);  // version, float, values, layers, in, out, height
  for (int c : {k, classes}) {  // c, u8, scale, zero, border rows, border columns
    u32(static_cast<uint32_t>(c));
    u32(0);
    const float one = 1.0f;
    put(&one, 4);
    u32(0);
    u32(0);
    u32(0);
  }
  const int32_t fields[20] = {kKindConv, 0, 1, -1, 1, 1, 1, 1, 0, 0, 0, 0, k, classes, 0, 1, 1, 1, 0, 0};
  put(fields, sizeof fields);
  for (size_t i = 0; i < cells; ++i) {
    __half_raw r;
    std::memcpy(&r.x, b + kHeader + 2 * i, 2);
    const float w = __half2float(__half(r));
    put(&w, 4);
  }
  put(b + kHeader + cells * 2, static_cast<size_t>(classes) * 4);
  return CREC_OK;
}

int crec_head_sweep(int device, int precision, const void* model, size_t model_bytes, int frames, const void* x,
                    int32_t* ids, float* probs, float* logits, int repeat, double* ms) {
  if (!model || !x || !ids || !probs || !ms || frames <= 0 || frames > (1 << 24) || repeat < 1 ||
      (precision != CREC_INT8 && precision != CREC_FP16))
    return CREC_E_INVALID;
  std::unique_ptr<crec_handle, void (*)(crec_handle*)> hold(new crec_handle(), [](crec_handle* p) {
    free_all(p);
    delete p;
  });
  crec_handle* h = hold.get();
  long long cols = 0;
  int rc = open_head(h, device, precision, model, model_bytes, frames, &cols);
  if (rc) return rc;
  const Layer& l = h->l[1];
  const Value& xv = h->v[l.in];
  const int classes = h->v[l.out].c;
  const size_t row = static_cast<size_t>(xv.cp) * h->eb;  // a frame's bytes
  CK(cudaMemcpy(xv.base + static_cast<long long>(xv.ph) * xv.pitch + static_cast<long long>(h->gap) * row, x,
                row * frames, cudaMemcpyHostToDevice));
  float* keep = h->d_logits;
  h->d_logits = nullptr;  // the timed launches write no logits
  if ((rc = launch_head(h, 1, cols))) return rc;  // warm-up
  CK(cudaStreamSynchronize(h->stream));
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  CK(cudaEventCreate(&e0));
  CK(cudaEventCreate(&e1));
  CK(cudaEventRecord(e0, h->stream));
  for (int r = 0; r < repeat && rc == CREC_OK; ++r) rc = launch_head(h, 1, cols);
  CK(cudaEventRecord(e1, h->stream));
  CK(cudaEventSynchronize(e1));
  float t = 0.0f;
  cudaEventElapsedTime(&t, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  h->d_logits = keep;
  if (rc) return rc;
  if (logits && (rc = launch_head(h, 1, cols))) return rc;  // once more, keeping the logits
  CK(cudaStreamSynchronize(h->stream));
  int err = 0;
  CK(cudaMemcpy(&err, h->d_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (err) return CREC_E_TIMEOUT;
  *ms = static_cast<double>(t) / repeat;
  CK(cudaMemcpy(ids, h->d_frame_id + h->gap, sizeof(int32_t) * frames, cudaMemcpyDeviceToHost));
  CK(cudaMemcpy(probs, h->d_frame_prob + h->gap, sizeof(float) * frames, cudaMemcpyDeviceToHost));
  if (logits)
    CK(cudaMemcpy(logits, h->d_logits + static_cast<size_t>(h->gap) * classes, sizeof(float) * frames * classes,
                  cudaMemcpyDeviceToHost));
  return CREC_OK;
}

int crec_conv_sweep(int device, int precision, const void* model, size_t model_bytes, int n, int h_in, int w,
                    const void* x, void* y, int repeat, double* ms) {
  if (!model || !x || !y || !ms || n <= 0 || h_in <= 0 || h_in > 64 || w <= 0 || repeat < 1 ||
      (precision != CREC_INT8 && precision != CREC_FP16))
    return CREC_E_INVALID;
  std::unique_ptr<crec_handle, void (*)(crec_handle*)> hold(new crec_handle(), [](crec_handle* p) {
    free_all(p);
    delete p;
  });
  crec_handle* h = hold.get();
  long long cols = 0;
  int rc = open_layer(h, device, precision, model, model_bytes, n, h_in, w, &cols);
  if (rc) return rc;
  const Layer& l = h->l[1];
  const Value& xv = h->v[l.in];
  const Value& yv = h->v[l.out];
  const size_t xrow = static_cast<size_t>(w) * xv.c * h->eb;
  for (int i = 0; i < n; ++i) {  // line i at input columns [gap + i (w + gap), + w)
    const long long seg = h->gap + static_cast<long long>(i) * (w + h->gap);
    CK(cudaMemcpy2D(xv.base + static_cast<long long>(xv.ph) * xv.pitch + seg * xv.cp * h->eb, xv.pitch,
                    static_cast<const uint8_t*>(x) + static_cast<size_t>(i) * h_in * xrow, xrow, xrow, h_in,
                    cudaMemcpyHostToDevice));
  }
  if ((rc = launch_conv(h, 1, cols))) return rc;  // warm-up
  CK(cudaStreamSynchronize(h->stream));
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  CK(cudaEventCreate(&e0));
  CK(cudaEventCreate(&e1));
  CK(cudaEventRecord(e0, h->stream));
  for (int r = 0; r < repeat && rc == CREC_OK; ++r) rc = launch_conv(h, 1, cols);
  CK(cudaEventRecord(e1, h->stream));
  CK(cudaEventSynchronize(e1));
  float t = 0.0f;
  cudaEventElapsedTime(&t, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (rc) return rc;
  int err = 0;
  CK(cudaMemcpy(&err, h->d_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (err) return CREC_E_TIMEOUT;
  *ms = static_cast<double>(t) / repeat;
  const int ow = w >> yv.shift;
  const size_t yrow = static_cast<size_t>(ow) * yv.c * h->eb;
  for (int i = 0; i < n; ++i) {
    const long long seg = (h->gap + static_cast<long long>(i) * (w + h->gap)) >> yv.shift;
    CK(cudaMemcpy2D(static_cast<uint8_t*>(y) + static_cast<size_t>(i) * yv.h * yrow, yrow,
                    yv.base + static_cast<long long>(yv.ph) * yv.pitch + seg * yv.cp * h->eb, yv.pitch, yrow, yv.h,
                    cudaMemcpyDeviceToHost));
  }
  return CREC_OK;
}

int crec_mma_peak(int device, int precision, int n, int iters, double* tera_ops) {
  if (!tera_ops || n < 16 || n > 256 || n % 16 || iters < 1 || (precision != CREC_INT8 && precision != CREC_FP16))
    return CREC_E_INVALID;
  if (cudaSetDevice(device) != cudaSuccess) return CREC_E_CUDA;
  cudaDeviceProp prop{};
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return CREC_E_CUDA;
  if (prop.major != 10) return CREC_E_INVALID;
  int* err = nullptr;
  if (cudaMalloc(&err, sizeof(int)) != cudaSuccess) return CREC_E_NOMEM;
  cudaMemset(err, 0, sizeof(int));
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  const int smem = kPeakSmem;
  auto launch = [&](int it) {
    if (precision == CREC_INT8) {
      cudaFuncSetAttribute(mma_peak_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      mma_peak_kernel<true><<<prop.multiProcessorCount, 128, smem>>>(n, it, err);
    } else {
      cudaFuncSetAttribute(mma_peak_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      mma_peak_kernel<false><<<prop.multiProcessorCount, 128, smem>>>(n, it, err);
    }
  };
  launch(16);  // warm-up
  cudaEventRecord(e0);
  launch(iters);
  cudaEventRecord(e1);
  int rc = cudaEventSynchronize(e1) == cudaSuccess ? CREC_OK : CREC_E_CUDA;
  int h_err = 0;
  if (rc == CREC_OK && cudaMemcpy(&h_err, err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) rc = CREC_E_CUDA;
  if (rc == CREC_OK && cudaGetLastError() != cudaSuccess) rc = CREC_E_CUDA;
  if (rc == CREC_OK && h_err) rc = CREC_E_TIMEOUT;
  float ms = 0.0f;
  cudaEventElapsedTime(&ms, e0, e1);
  // multiply-adds an MMA: 128 x n x K, K = 32 bytes (32 int8, 16 fp16)
  const double k = precision == CREC_INT8 ? 32.0 : 16.0;
  const double ops = 2.0 * 128.0 * n * k * 4.0 * iters * prop.multiProcessorCount;
  *tera_ops = rc == CREC_OK && ms > 0 ? ops / (ms * 1e-3) / 1e12 : 0.0;
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaFree(err);
  return rc;
}
