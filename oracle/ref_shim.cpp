// C entry points over the reference's own CPU line-recognition code, compiled from
// its sources (oracle/ref.mk) into oracle/_ref/libcarbon_ref.so.
//
// TEST INFRASTRUCTURE ONLY.  This file is the checker, never the product: only
// tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load the
// library it builds.  It calls the reference's functions unchanged:
//   crop_region / resample_gray / crop_lines / finish_crop / crop_ground
//       carbon/src/lines.cpp:33, :252, :279, :311, :269
//   ctc_greedy / ctc_collapse                      carbon/src/lines.cpp:357, :331
//   cpu::detail::exp_neg                           carbon/src/cpu/kernels.h:226
//   open_session(kNative) -> NativeSession::run    carbon/src/net/net.cpp:1186-1214
//   onnx::cut                                      carbon/src/net/onnx.h:87
// and adds a threaded timing harness laid out like the reference's CPU engine
// (one single-threaded native session per pinned worker, carbon/src/engine.cpp:1297).
#include <pthread.h>
#include <sched.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdint>
#include <cstring>
#include <exception>
#include <memory>
#include <string>
#include <thread>
#include <vector>

#include "carbon/cpu.h"
#include "carbon/error.h"
#include "carbon/lines.h"
#include "carbon/session.h"
#include "carbon/tensor.h"
#include "cpu/kernels.h"
#include "net/onnx.h"

namespace {

thread_local std::string g_error;

int fail(const std::exception& e) {
  g_error = e.what();
  return -1;
}

struct RefRule {
  int height, width_step, frame_px;
  double pad_v, pad_h;
  int flip_margin, flip_needs_dark;
};

carbon::CropRule rule_of(const RefRule* r) {
  carbon::CropRule c;
  if (!r) return c;
  c.height = r->height;
  c.width_step = r->width_step;
  c.frame_px = r->frame_px;
  c.pad_v = r->pad_v;
  c.pad_h = r->pad_h;
  c.flip_margin = r->flip_margin;
  c.flip_needs_dark = r->flip_needs_dark != 0;
  return c;
}

}  // namespace

extern "C" {

const char* ref_last_error() { return g_error.c_str(); }

void ref_default_rule(RefRule* r) {
  const carbon::CropRule c;
  r->height = c.height;
  r->width_step = c.width_step;
  r->frame_px = c.frame_px;
  r->pad_v = c.pad_v;
  r->pad_h = c.pad_h;
  r->flip_margin = c.flip_margin;
  r->flip_needs_dark = c.flip_needs_dark ? 1 : 0;
}

int ref_crop_region(const double* box, const RefRule* rule, double* region, int* width) {
  try {
    const carbon::CropRegion c = carbon::crop_region({box[0], box[1], box[2], box[3]}, rule_of(rule));
    region[0] = c.x0;
    region[1] = c.y0;
    region[2] = c.x1;
    region[3] = c.y1;
    *width = c.width;
    return 0;
  } catch (const std::exception& e) {
    return fail(e);
  }
}

int ref_resample_gray(const uint8_t* img, int w, int h, int64_t stride, double x0, double y0, double x1, double y1,
                      int ow, int oh, uint8_t* out, int64_t os, int scalar) {
  try {
    const carbon::GrayView v{img, w, h, stride};
    carbon::resample_gray(v, x0, y0, x1, y1, ow, oh, out, os,
                          scalar ? carbon::cpu::Isa::kScalar : carbon::cpu::best_isa());
    return 0;
  } catch (const std::exception& e) {
    return fail(e);
  }
}

int ref_crop_lines(const uint8_t* page, int w, int h, int64_t stride, const double* boxes, int n, int out_width,
                   uint8_t* out, int32_t* widths, const RefRule* rule) {
  try {
    const carbon::GrayView v{page, w, h, stride};
    std::vector<carbon::LineBox> b(static_cast<size_t>(n));
    for (int i = 0; i < n; ++i) b[i] = {boxes[4 * i], boxes[4 * i + 1], boxes[4 * i + 2], boxes[4 * i + 3]};
    carbon::crop_lines(v, b, out_width, out, std::span<int32_t>(widths, static_cast<size_t>(n)), rule_of(rule));
    return 0;
  } catch (const std::exception& e) {
    return fail(e);
  }
}

int ref_finish_crop(uint8_t* crop, int w, int out_width, const RefRule* rule) {
  try {
    carbon::finish_crop(crop, w, out_width, rule_of(rule));
    return 0;
  } catch (const std::exception& e) {
    return fail(e);
  }
}

int ref_crop_ground(const uint8_t* crop, int w, int h, int64_t stride) { return carbon::crop_ground(crop, w, h, stride); }

int ref_light_on_dark(const uint8_t* crop, int w, int h, int64_t stride, int margin) {
  return carbon::light_on_dark(crop, w, h, stride, margin) ? 1 : 0;
}

float ref_exp_neg(float x) { return carbon::cpu::detail::exp_neg(x); }

// carbon::load_ctc_head on a file: its classes and k, and up to `cap` weights (float16 bits) and
// `classes` biases (or -1, the reason in ref_last_error()).
int ref_load_ctc_head(const char* path, int* classes, int* k, uint16_t* weight, float* bias, int64_t cap) {
  try {
    const carbon::CtcHead hd = carbon::load_ctc_head(path);
    *classes = hd.classes;
    *k = hd.k;
    const size_t n = std::min<size_t>(hd.weight.size(), static_cast<size_t>(std::max<int64_t>(cap, 0)));
    std::memcpy(weight, hd.weight.data(), n * 2);
    if (static_cast<int64_t>(hd.weight.size()) <= cap) std::memcpy(bias, hd.bias.data(), hd.bias.size() * 4);
    return 0;
  } catch (const std::exception& e) {
    return fail(e);
  }
}

// cpu::ctc_topk (what carbon::frame_candidates calls) on one line's logits [classes][frames].
int ref_ctc_topk(const float* logits, int classes, int frames, int t_n, int k, int32_t* ids, float* logp, float* blank) {
  try {
    carbon::cpu::ctc_topk(logits, classes, frames, t_n, k, ids, logp, blank);
    return 0;
  } catch (const std::exception& e) {
    return fail(e);
  }
}

// ctc_greedy: per line its count, and up to `cap` ids, frames and probs at line i * cap.
int ref_ctc_greedy(const float* logits, int n, int classes, int frames, const int32_t* lengths, int cap,
                   int32_t* counts, int32_t* ids, int32_t* frame_of, float* probs) {
  try {
    const auto lines = carbon::ctc_greedy(logits, n, classes, frames,
                                          std::span<const int32_t>(lengths, static_cast<size_t>(n)));
    for (int i = 0; i < n; ++i) {
      const carbon::CtcLine& l = lines[i];
      const int k = static_cast<int>(l.ids.size());
      counts[i] = k;
      for (int j = 0; j < std::min(k, cap); ++j) {
        ids[static_cast<size_t>(i) * cap + j] = l.ids[j];
        frame_of[static_cast<size_t>(i) * cap + j] = l.frames[j];
        probs[static_cast<size_t>(i) * cap + j] = l.probs[j];
      }
    }
    return 0;
  } catch (const std::exception& e) {
    return fail(e);
  }
}

int ref_ctc_collapse(const int32_t* arg, const float* prob, int n, int frames, const int32_t* lengths, int cap,
                     int32_t* counts, int32_t* ids, int32_t* frame_of, float* probs) {
  try {
    const auto lines =
        carbon::ctc_collapse(arg, prob, n, frames, std::span<const int32_t>(lengths, static_cast<size_t>(n)));
    for (int i = 0; i < n; ++i) {
      const carbon::CtcLine& l = lines[i];
      const int k = static_cast<int>(l.ids.size());
      counts[i] = k;
      for (int j = 0; j < std::min(k, cap); ++j) {
        ids[static_cast<size_t>(i) * cap + j] = l.ids[j];
        frame_of[static_cast<size_t>(i) * cap + j] = l.frames[j];
        probs[static_cast<size_t>(i) * cap + j] = l.probs[j];
      }
    }
    return 0;
  } catch (const std::exception& e) {
    return fail(e);
  }
}

// A native session on a model file (or on `bytes`, a model the caller cut), kernels of `isa` ("" the best).
void* ref_open(const char* path, const char* isa, const char* bytes, size_t len) {
  try {
    carbon::SessionOptions o;
    o.threads = 1;
    if (isa) o.isa = isa;
    if (bytes) o.model_bytes = std::make_shared<const std::string>(bytes, len);
    return carbon::open_session(carbon::Backend::kNative, path, o).release();
  } catch (const std::exception& e) {
    fail(e);
    return nullptr;
  }
}

void ref_close(void* s) { delete static_cast<carbon::Session*>(s); }

// One run on x [n, c, h, w]: its first output into `out` (at most cap floats), its shape into shape[0..rank).
int ref_run(void* s, const float* x, int n, int c, int h, int w, float* out, int64_t cap, int64_t* shape,
            int* rank) {
  try {
    auto* session = static_cast<carbon::Session*>(s);
    carbon::Tensor t = carbon::Tensor::empty(carbon::DType::kFloat32, {n, c, h, w});
    std::memcpy(t.raw(), x, t.bytes());
    std::vector<carbon::Tensor> in;
    in.push_back(std::move(t));
    const std::vector<carbon::Tensor> o = session->run(in);
    const carbon::Tensor& y = o.at(0);
    *rank = static_cast<int>(y.shape().size());
    for (int i = 0; i < *rank; ++i) shape[i] = y.shape()[i];
    if (y.size() > cap) throw carbon::Error("ref_run: output of " + std::to_string(y.size()) + " floats, room for " +
                                            std::to_string(cap));
    std::memcpy(out, y.raw(), y.bytes());
    return 0;
  } catch (const std::exception& e) {
    return fail(e);
  }
}

// The model file cut at tensor `output` (float, shape dims[0..ndims), -1 free): its bytes, freed by ref_free.
int ref_cut(const char* path, const char* output, const int64_t* dims, int ndims, char** bytes, size_t* len) {
  try {
    FILE* f = std::fopen(path, "rb");
    if (!f) throw carbon::Error(std::string("cannot read ") + path);
    std::string model;
    char buf[1 << 16];
    size_t got;
    while ((got = std::fread(buf, 1, sizeof buf, f)) > 0) model.append(buf, got);
    std::fclose(f);
    const std::string cut = carbon::onnx::cut(model, output, carbon::onnx::kFloat,
                                              std::vector<int64_t>(dims, dims + ndims));
    *bytes = static_cast<char*>(std::malloc(cut.size()));
    std::memcpy(*bytes, cut.data(), cut.size());
    *len = cut.size();
    return 0;
  } catch (const std::exception& e) {
    return fail(e);
  }
}

void ref_free(void* p) { std::free(p); }

// The CPU baseline: `threads` workers, each pinned to core (first_cpu + worker) and holding its own
// single-threaded native session (the reference CPU engine's layout), run the batches of crops
// given (batch b: rows [row0[b], row0[b] + count[b]) of `crops`, each 32 x width[b] ink values, stored
// at crop_offset[b] floats), batches dealt round-robin, for `rounds` passes; then ctc_greedy on each
// batch's logits (the reference's CpuModels::recognize minus the crop, carbon/src/pipeline.cpp:138-162).
// Returns the wall seconds of the timed passes (after one untimed pass), or < 0 on an error.
double ref_bench_batches(const char* model, const char* isa, int threads, int first_cpu, int batches,
                         const float* crops, const int64_t* crop_offset, const int32_t* count, const int32_t* width,
                         const int32_t* lengths_all, int height, int rounds) {
  try {
    std::vector<std::unique_ptr<carbon::Session>> sessions(static_cast<size_t>(threads));
    for (int t = 0; t < threads; ++t) {
      carbon::SessionOptions o;
      o.threads = 1;
      if (isa) o.isa = isa;
      sessions[t] = carbon::open_session(carbon::Backend::kNative, model, o);
    }
    std::vector<int64_t> line0(static_cast<size_t>(batches) + 1, 0);
    for (int b = 0; b < batches; ++b) line0[b + 1] = line0[b] + count[b];
    std::atomic<int> errors{0};
    auto work = [&](int t, int passes) {
      cpu_set_t set;
      CPU_ZERO(&set);
      CPU_SET(first_cpu + t, &set);
      pthread_setaffinity_np(pthread_self(), sizeof set, &set);
      try {
        for (int r = 0; r < passes; ++r) {
          for (int b = t; b < batches; b += threads) {
            carbon::Tensor x = carbon::Tensor::empty(carbon::DType::kFloat32, {count[b], 1, height, width[b]});
            std::memcpy(x.raw(), crops + crop_offset[b], x.bytes());
            std::vector<carbon::Tensor> in;
            in.push_back(std::move(x));
            const std::vector<carbon::Tensor> o = sessions[t]->run(in);
            const carbon::Shape& s = o[0].shape();
            const auto lines = carbon::ctc_greedy(o[0].data<float>().data(), count[b], static_cast<int>(s[1]),
                                                  static_cast<int>(s[2]),
                                                  std::span<const int32_t>(lengths_all + line0[b],
                                                                           static_cast<size_t>(count[b])));
            if (lines.size() != static_cast<size_t>(count[b])) errors++;
          }
        }
      } catch (...) {
        errors++;
      }
    };
    auto run_all = [&](int passes) {
      std::vector<std::thread> pool;
      for (int t = 0; t < threads; ++t) pool.emplace_back(work, t, passes);
      for (auto& th : pool) th.join();
    };
    run_all(1);  // warm-up: every session's buffers sized
    const auto t0 = std::chrono::steady_clock::now();
    run_all(rounds);
    const double secs = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (errors) throw carbon::Error("ref_bench_batches: a worker failed");
    return secs;
  } catch (const std::exception& e) {
    fail(e);
    return -1.0;
  }
}

// The CPU baseline on pages, as the reference's CPU device recognizes a run
// (CpuModels::recognize, carbon/src/pipeline.cpp:138-162): per batch (lines of one bucket width,
// at most 256, contiguous in the arrays), crop_lines per run of lines of one page, the ink map
// 1 - p / 255, the native session, ctc_greedy with lengths min(frames, width / 4).  `threads`
// pinned workers (cores first_cpu...), each with its own single-threaded session, take batches
// round-robin.  One untimed pass, then `rounds` timed passes; returns their wall seconds.
double ref_bench_pages(const char* model, const char* isa, int threads, int first_cpu, int npages,
                       const uint8_t* const* page_data, const int32_t* page_w, const int32_t* page_h,
                       const int64_t* page_stride, int batches, const int32_t* batch_start,
                       const int32_t* batch_count, const int32_t* batch_bw, const int32_t* page_of,
                       const double* boxes, int rounds, int64_t* lines_done) {
  try {
    std::vector<std::unique_ptr<carbon::Session>> sessions(static_cast<size_t>(threads));
    for (int t = 0; t < threads; ++t) {
      carbon::SessionOptions o;
      o.threads = 1;
      if (isa) o.isa = isa;
      sessions[t] = carbon::open_session(carbon::Backend::kNative, model, o);
    }
    std::atomic<int> errors{0};
    std::atomic<int64_t> done{0};
    const carbon::CropRule rule;
    auto work = [&](int t, int passes) {
      cpu_set_t set;
      CPU_ZERO(&set);
      CPU_SET(first_cpu + t, &set);
      pthread_setaffinity_np(pthread_self(), sizeof set, &set);
      try {
        std::vector<uint8_t> crops;
        std::vector<int32_t> widths;
        for (int r = 0; r < passes; ++r) {
          for (int b = t; b < batches; b += threads) {
            const int a0 = batch_start[b], m = batch_count[b], bw = batch_bw[b], h = rule.height;
            crops.assign(static_cast<size_t>(m) * h * bw, 0);
            widths.assign(m, 0);
            for (int i = 0; i < m;) {
              int e = i + 1;
              while (e < m && page_of[a0 + e] == page_of[a0 + i]) ++e;
              const int pg = page_of[a0 + i];
              const carbon::GrayView v{page_data[pg], page_w[pg], page_h[pg], page_stride[pg]};
              std::vector<carbon::LineBox> bx;
              for (int k = i; k < e; ++k) {
                const double* q = boxes + 4 * static_cast<size_t>(a0 + k);
                bx.push_back({q[0], q[1], q[2], q[3]});
              }
              carbon::crop_lines(v, bx, bw, crops.data() + static_cast<size_t>(i) * h * bw,
                                 std::span<int32_t>(widths.data() + i, static_cast<size_t>(e - i)), rule);
              i = e;
            }
            carbon::Tensor x = carbon::Tensor::empty(carbon::DType::kFloat32, {m, 1, h, bw});
            float* px = x.data<float>().data();
            for (size_t i = 0; i < crops.size(); ++i) px[i] = 1.0f - crops[i] / 255.0f;
            std::vector<carbon::Tensor> in;
            in.push_back(std::move(x));
            const std::vector<carbon::Tensor> o = sessions[t]->run(in);
            const carbon::Shape& s = o[0].shape();
            std::vector<int32_t> lengths(m);
            for (int i = 0; i < m; ++i) lengths[i] = std::min<int32_t>(static_cast<int32_t>(s[2]), widths[i] / rule.frame_px);
            const auto lines = carbon::ctc_greedy(o[0].data<float>().data(), m, static_cast<int>(s[1]),
                                                  static_cast<int>(s[2]), lengths);
            if (lines.size() != static_cast<size_t>(m)) errors++;
            done += m;
          }
        }
      } catch (...) {
        errors++;
      }
    };
    auto run_all = [&](int passes) {
      std::vector<std::thread> pool;
      for (int t = 0; t < threads; ++t) pool.emplace_back(work, t, passes);
      for (auto& th : pool) th.join();
    };
    run_all(1);
    done = 0;
    const auto t0 = std::chrono::steady_clock::now();
    run_all(rounds);
    const double secs = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (errors) throw carbon::Error("ref_bench_pages: a worker failed");
    if (lines_done) *lines_done = done;
    return secs;
  } catch (const std::exception& e) {
    fail(e);
    return -1.0;
  }
}

}  // extern "C"
