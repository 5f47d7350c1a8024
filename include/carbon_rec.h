/* carbon_rec: Carbon-OCR's line recognition (crop, the recognizer, greedy CTC) on B200
 * (sm_100a), behind a C ABI.
 *
 * These entry points are what a device behind the reference's recognizer-backend interface,
 * carbon::PipelineModels (carbon/include/carbon/pipeline.h:94-142 of the reference), binds:
 *
 *   crec_open / crec_close        the device's construction from a set's recognizer file and
 *                                 the crop rule (cuda_pipeline_models, pipeline.h:199-200;
 *                                 CudaModels, carbon/src/cuda/pipeline_cuda.cpp:146)
 *   crec_set_pages                PipelineModels::set_pages (pipeline.h:120)
 *   crec_prefetch_pages           PipelineModels::prefetch_pages (pipeline.h:124)
 *   crec_recognize                PipelineModels::recognize (pipeline.h:131-132)
 *   crec_is_broken                PipelineModels::broken (pipeline.h:116)
 *   crec_width_bucket             carbon::width_bucket (carbon/src/engine.cpp:669-675)
 *   crec_crop_region              carbon::crop_region (carbon/src/lines.cpp:33)
 *   crec_recognize_lines          the recognize stage's bucketing and runs
 *                                 (carbon/src/pipeline.cpp:536-603) done on the device side:
 *                                 any number of lines in as few launches as fit
 *
 * Plain pointers and sizes only.  Every call returns a status (CREC_OK or an error code);
 * no exception crosses the ABI; crec_last_error() gives the message.  A handle drives one
 * GPU and is not safe to call from two threads at once (the reference's recognize stage
 * calls its device from one thread, pipeline.h:92-93); open one handle per GPU.  A handle
 * starts threads of its own when it first needs them and ends them at crec_close: up to 8 that
 * stage pageable page rows into pinned chunks (half the host's CPUs, at most 8), one uploader
 * for crec_prefetch_pages, and up to 7 that lay out a call's runs of 2,048 lines or more; they
 * sleep or wait on the GPU between calls.
 */
#ifndef CARBON_REC_H_
#define CARBON_REC_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define CREC_API __attribute__((visibility("default")))
#else
#define CREC_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define CREC_OK 0
#define CREC_E_INVALID 1 /* an argument is out of its range */
#define CREC_E_NOMEM 2   /* device or pinned host memory could not be had */
#define CREC_E_CUDA 3    /* a CUDA call failed; the handle is still usable */
#define CREC_E_STICKY 4  /* a sticky CUDA error: this process can use the GPU no more (crec_is_broken) */
#define CREC_E_TIMEOUT 5 /* a kernel's bounded wait ran out; the run's results are not valid */
#define CREC_E_MODEL 6   /* the model blob is not one this build runs */
#define CREC_E_RANGE 7   /* a crop wider than its batch, or more lines or columns than configured */

#define CREC_INT8 0 /* the Q/DQ recognizer: int8 weights, uint8 activations, int32 sums */
#define CREC_FP16 1 /* the float recognizer: float16 weights and activations, float32 sums */

typedef struct crec_handle crec_handle;

/* carbon::CropRule (carbon/include/carbon/lines.h:23-37). */
typedef struct crec_crop_rule {
  int height;     /* px; 32 */
  int width_step; /* 8 */
  int frame_px;   /* 4 */
  double pad_v;   /* 0.2 */
  double pad_h;   /* 0.3 */
  int flip_margin;     /* 48; 0: never flip */
  int flip_needs_dark; /* 1 */
} crec_crop_rule;

typedef struct crec_config {
  int precision;   /* CREC_INT8 or CREC_FP16 */
  int device;      /* CUDA device ordinal */
  int max_lines;   /* lines one recognize call may hold (the pipeline's line_batch, or more) */
  int max_width;   /* the widest bucket, px (the reference's ladder ends at 2048) */
  int64_t max_columns; /* columns of crop width (plus gaps) one run holds on the device; 0: from the two above */
  int max_pages;       /* pages a set_pages call may hold */
  int64_t max_page_bytes; /* bytes of pages held on the device; 0: max_pages letter pages at 200 dpi */
  crec_crop_rule crop;
  const void* model;   /* the recognizer as a "CRECMDL1" blob (carbon_rec/netdef.py): the Q/DQ file's for
                          CREC_INT8, the float file's for CREC_FP16 (its weights rounded to float16) */
  size_t model_bytes;
} crec_config;

/* carbon::GrayView (lines.h:56-60): a grayscale page, paper 255, rows `stride` bytes apart. */
typedef struct crec_page {
  const uint8_t* data;
  int width, height;
  int64_t stride;
} crec_page;

/* carbon::RowRuns (pipeline.h:88-90): the rows [runs[2i], runs[2i+1]) a page's crops read; count 0: all. */
typedef struct crec_row_runs {
  const int32_t* runs;
  int count;
} crec_row_runs;

/* carbon::LineBox (lines.h:40-42): page pixels, x right, y down. */
typedef struct crec_box {
  double x0, y0, x1, y1;
} crec_box;

/* A run's decodings (carbon::CtcLine, lines.h:107-112), in arrays the caller owns. */
typedef struct crec_lines {
  int32_t* counts;  /* [n] characters of line i */
  int32_t* lengths; /* [n] frames read: min(frames, crop width / frame_px) */
  int32_t* offsets; /* [n] where line i's characters start in ids, frames and probs */
  int32_t* ids;     /* class ids, blanks dropped and repeats collapsed */
  int32_t* frames;  /* each character's first frame */
  float* probs;     /* each character's highest softmax probability over its run */
  int64_t capacity; /* room in ids, frames and probs (sum over lines of bw / frame_px always suffices) */
  int64_t total;    /* characters written */
} crec_lines;

CREC_API int crec_open(const crec_config* config, crec_handle** out);
CREC_API int crec_close(crec_handle* h);
CREC_API const char* crec_last_error(const crec_handle* h);
/* Whether a sticky error left the GPU unusable for this process (PipelineModels::broken). */
CREC_API int crec_is_broken(const crec_handle* h);

/* The pages the recognize calls that follow crop from, on the GPU (only rows[i]'s runs copied
 * where given): the pages a prefetch_pages call gave already (same pointers and sizes), else
 * uploaded now. The copies run on their own stream; the recognize work waits for them on the
 * device. The pages must stay alive and unchanged until the next set_pages or prefetch_pages
 * call returns (or crec_close), as the reference's contract has them (pipeline.h:118-120). */
CREC_API int crec_set_pages(crec_handle* h, const crec_page* pages, int n, const crec_row_runs* rows);
/* The next group's pages, given while the current group is read (pipeline.h:121-124): uploaded
 * now into the second page buffer on the copy stream, beside the current group's runs; the
 * set_pages with these same pages then only switches buffers. Same lifetime rule. */
CREC_API int crec_prefetch_pages(crec_handle* h, const crec_page* pages, int n, const crec_row_runs* rows);
/* Pages already in this handle's GPU memory (data are device pointers): used in place. */
CREC_API int crec_set_pages_device(crec_handle* h, const crec_page* pages, int n);

/* PipelineModels::recognize: the lines boxes[i] of page page_of[i], cropped at bucket width bw
 * (a multiple of the crop rule's width step), decoded; lengths[i] = min(bw / frame_px, crop
 * width / frame_px). CREC_E_RANGE if a crop is wider than bw. */
CREC_API int crec_recognize(crec_handle* h, const int32_t* page_of, const crec_box* boxes, int n, int bw, crec_lines* out);
/* Any number of lines, each at its own bucket width (bw[i]; null: crec_width_bucket of its crop
 * width), in as few device runs as the configured columns allow; results as crec_recognize. */
CREC_API int crec_recognize_lines(crec_handle* h, const int32_t* page_of, const crec_box* boxes, const int32_t* bw, int n,
                         crec_lines* out);

/* Crops given ready ([n][crop height][pitch] bytes, line i's first bw[i] columns already finished
 * and padded, as crop_lines gives them; widths[i] its own crop width): the recognizer and CTC
 * on them, as the reference's CPU device runs its session on crop_lines' output
 * (carbon/src/pipeline.cpp:138-162).  At most max_lines; pitch at most max_width. */
CREC_API int crec_recognize_crops(crec_handle* h, const uint8_t* crops, int pitch, const int32_t* widths, const int32_t* bw,
                         int n, crec_lines* out);

/* carbon::cuda::ctc_greedy (carbon/include/carbon/cuda.h:58-62 of the reference): greedy CTC
 * decoding of device logits [n][classes][frames] (float32), each line's first lengths[i] frames
 * (a host array), queued on `stream` (a cudaStream_t; null the default stream) and waited for.
 * Ids, frames and probabilities are carbon::ctc_greedy's, bit for bit.  Its scratch is allocated
 * and freed on the stream by the call.  No handle: a message for an error goes to error[0,
 * error_size) (may be null).  out->lengths gets min(lengths[i], frames). */
CREC_API int crec_ctc_greedy(const float* logits, int n, int classes, int frames, const int32_t* lengths,
                             crec_lines* out, void* stream, char* error, size_t error_size);

/* crec_ctc_greedy without allocating: for callers that cannot have a library call cudaMalloc or
 * cudaMallocAsync -- a process whose device memory all belongs to its own allocator (a framework's
 * caching allocator, an arena reserved at start-up) or a serving path that fixed its memory before
 * it started.  No counterpart in the reference.  Everything is in device memory and queued on
 * `stream` without waiting: logits [n][classes][frames] (float32), lengths [n], and the outputs
 * counts [n] and ids, starts, probs [n][frames] (line i's characters at [i * frames, i * frames +
 * counts[i])), the same values as crec_ctc_greedy's.  With n > 0, lengths and counts are always
 * required; logits, ids, starts and probs when frames > 0 (CREC_E_INVALID otherwise).  With
 * frames == 0 no kernel runs: counts is cleared on `stream`.  The per-frame scratch is a 4 MiB device
 * array inside this library: n x frames may be at most 524,288 (CREC_E_RANGE beyond, nothing
 * queued).  Each call on a device uses the same array, so calls whose work overlaps on the GPU
 * (two streams, two threads) race: order them on one stream.  The first call on each device looks
 * the array's address up (cudaGetSymbolAddress, with that device current): make it before any
 * stream capture. */
CREC_API int crec_ctc_greedy_noalloc(const float* logits, int n, int classes, int frames, const int32_t* lengths,
                                     int32_t* counts, int32_t* ids, int32_t* starts, float* probs, void* stream,
                                     char* error, size_t error_size);

CREC_API int crec_width_bucket(int crop_width);
/* carbon::crop_region: the page rectangle a box's crop resamples (region[4]: x0, y0, x1, y1) and
 * the crop's width. */
CREC_API int crec_crop_region(const crec_box* box, const crec_crop_rule* rule, double* region, int* width);

/* The beam's candidates (carbon::PipelineModels::candidates, carbon/include/carbon/pipeline.h:133-141;
 * carbon::frame_candidates, carbon/include/carbon/beam.h:40-51) of lines rows[0..n) of the last
 * recognize call (indices into its lines; each must lie in the call's last run -- a call of more
 * lines or columns than a run holds keeps only its last run's head input; ask before the next
 * call).  topk is clamped to [0, min(16, classes - 1)], as the reference's GPU device clamps it,
 * and *k gets the value used.  frames[j] gets line j's frame count t_j (its length, as the call
 * returned it), and the lines' frames are packed in row order, line j's from the sum of the earlier
 * t's: for each frame its k likeliest classes but the blank, best first (ties to the lower id),
 * ids[f * k + q] and their log-probabilities logp[f * k + q], and the blank's, blank[f]; each the
 * logit less the frame's best and ln of the class-order sum of exp(logit - best), as the CPU
 * reference's ctc_topk computes them (the INT8 logits are the run's own codes, made again on the
 * GPU from the head's input; FP16 logits within about 1e-3 of the fused head's).  capacity: the
 * frames the arrays hold (ids and logp capacity * k entries). */
CREC_API int crec_candidates(crec_handle* h, const int32_t* rows, int n, int topk, int32_t* k, int32_t* frames,
                             int32_t* ids, float* logp, float* blank, int64_t capacity);

/* What the last call did: device runs, kernel launches, bytes copied host -> device and back
 * (for crec_set_pages, the upload of the pages it took, whether it made that upload itself or a
 * crec_prefetch_pages made it); and the bytes copied each way since the handle was opened (every
 * page upload, prefetched or not, and every call's own copies). */
typedef struct crec_stats {
  int64_t runs, launches, h2d_bytes, d2h_bytes;
  int64_t h2d_total, d2h_total;
  int64_t wide_lines; /* the last call's lines resampled by the wide-reach path (past 15x or 1024 source rows) */
} crec_stats;
CREC_API int crec_last_stats(const crec_handle* h, crec_stats* out);

/* Per-kernel device times, measured with CUDA events around each launch on the handle's stream:
 * one entry per kernel kind (its name, launches, milliseconds summed, and algorithmic operations --
 * 2 x multiply-adds over the lines' own columns -- summed), totals since profiling was last
 * (re)started.  enable 1 starts (or restarts) profiling, 0 stops it, -1 leaves it as it is; out
 * (null: not read) gets up to `capacity` entries; returns the entries written. */
typedef struct crec_profile_entry {
  const char* kernel;
  int64_t launches;
  double ms;
  double ops;
} crec_profile_entry;
CREC_API int crec_profile(crec_handle* h, int enable, crec_profile_entry* out, int capacity);

/* The profile by layer: entry i for the model's layer i (0 the crop and stem, the last the head
 * with CTC; a Resize read in place has no launches), then one for the collapse; the same totals
 * crec_profile gathers, cleared and enabled by it.  Returns the entries written (at most
 * capacity), or a negative status.  No counterpart in the reference (a diagnostic). */
CREC_API int crec_profile_layers(crec_handle* h, crec_profile_entry* out, int capacity);

/* The tensor cores' dense rate, measured on GPU `device`: every SM issuing back-to-back
 * tcgen05.mma (M = 128, K = 32 bytes, N = n, 16..256) of `precision` (CREC_INT8: u8 x s8 -> s32;
 * CREC_FP16: f16 -> f32) from shared memory into TMEM, `iters` x 4 each. *tera_ops: 2 x
 * multiply-adds a second / 1e12. The roofline's denominator for this build's tensor kernels.
 * No counterpart in the reference (a measurement). */
CREC_API int crec_mma_peak(int device, int precision, int n, int iters, double* tera_ops);

/* Test hooks for the failure paths, armed for the next device run (no counterpart in the
 * reference).  CREC_INJECT_TIMEOUT: the run's first dense convolution loads nothing and every
 * wait of that launch gives up after 1 ms instead of 2 s, so its bounded waits run out: the
 * kernel ends, the run reports CREC_E_TIMEOUT, and the handle stays usable.  CREC_INJECT_STICKY:
 * once the run has completed, its completion check reports cudaErrorLaunchFailure (the error a
 * faulted kernel leaves), so the handle takes the sticky-error path: CREC_E_STICKY, then
 * crec_is_broken and CREC_E_STICKY from every later call. */
#define CREC_INJECT_TIMEOUT 1
#define CREC_INJECT_STICKY 2
CREC_API int crec_debug_inject(crec_handle* h, int what);

/* The kernel sweep (on the CPU the reference measures its GEMMs with
 * cli/main.cpp's bench_gemm): a blob's one dense convolution (its input value, the layer, its
 * output value; carbon_rec/model.py make_conv) run by this build's tcgen05 implicit-GEMM kernel,
 * set up as in a recognizer, on n inputs [h][w][c_in] (NHWC, each its own line with the zero
 * point -- a real 0 -- around it, as the reference's executor borders a batch): uint8 codes for
 * CREC_INT8, float16 for CREC_FP16; y gets [n][oh][ow][c_out] the same way.  *ms: the kernel's
 * mean device time over `repeat` launches after one warm-up (CUDA events).  Channel counts must
 * be multiples of 16.  No counterpart in the reference (a measurement and parity hook). */
CREC_API int crec_conv_sweep(int device, int precision, const void* model, size_t model_bytes, int n, int h, int w,
                             const void* x, void* y, int repeat, double* ms);

/* The head sweep (BASELINE.json config 4's head GEMM; the reference's GPU head is
 * carbon::cuda::ctc_head_argmax, carbon/include/carbon/cuda.h, tested in
 * tests/cpp/cuda_ctc_head_test.cpp): a blob's one 1x1 convolution, K channels to `classes`, run
 * as this build's fused head (tcgen05 GEMM, each frame's argmax and, for a frame whose best class
 * is not 0 -- the CTC blank --, its probability 1 / sum_c exp(logit_c - logit_best)) over `frames`
 * frames x [frames][K] (uint8 codes for CREC_INT8, float16 for CREC_FP16).  ids[frames] get the
 * first class of the highest logit, probs[frames] the probability (0 for blank frames); logits
 * (optional, [frames][classes]) each frame's logits as the head computed them (INT8: the
 * dequantized output codes).  K * element bytes must be a multiple of 16 and at most 1024.  *ms:
 * the mean device time of the head's launches (with the INT8 probability sums) over `repeat`
 * after one warm-up.  A measurement and parity hook. */
/* carbon::load_ctc_head (carbon/include/carbon/lines.h:120-135, carbon/src/lines.cpp:372-398): a
 * recognizer's last 1x1 convolution as the export writes it, <model>.head.bin ("CTCHEAD1", int32
 * classes, int32 k, the weight [classes][k] in float16, the bias [classes] in float32), checked as
 * the reference checks it (CREC_E_MODEL, the reason in `error`), made into this library's FP16
 * model blob of that one layer (for crec_head_sweep with CREC_FP16).  *blob_bytes gets the blob's
 * size; CREC_E_RANGE when blob is null or capacity is smaller. */
CREC_API int crec_ctc_head_blob(const void* file, size_t bytes, void* blob, size_t capacity, size_t* blob_bytes,
                                char* error, size_t error_size);
CREC_API int crec_head_sweep(int device, int precision, const void* model, size_t model_bytes, int frames,
                             const void* x, int32_t* ids, float* probs, float* logits, int repeat, double* ms);

/* The CUDA stream (a cudaStream_t) the handle's work runs on, for device-side timing. */
CREC_API void* crec_stream(crec_handle* h);

/* Test hooks: the last run's finished crops ([n][height][pitch] bytes, each line's first
 * bucket-width columns), and a network tensor of the last run (value index of the model
 * blob; each line's NHWC values without borders, lines one after another: uint8 for
 * CREC_INT8, float16 for CREC_FP16). */
CREC_API int crec_debug_crops(crec_handle* h, uint8_t* out, int pitch);
CREC_API int crec_debug_value(crec_handle* h, int value, void* out, int64_t capacity_bytes);
/* Test hook: the last run's logits, each line's [classes][bw / frame_px] floats one after another
 * (INT8: the uint8 logits' values, (q - zero) * scale, as the reference's output table gives them;
 * FP16: the FP32 sums).  out null arms it: the runs from then on write them (slower). */
CREC_API int crec_debug_logits(crec_handle* h, float* out, int64_t capacity);

#ifdef __cplusplus
}
#endif

#endif /* CARBON_REC_H_ */
