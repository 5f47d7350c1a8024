// Greedy CTC decoding of logits already in device memory: the unfused path
// (carbon::cuda::ctc_greedy, carbon/src/cuda/lines.cu:264-309 of the reference), for a
// recognizer whose last layer ran elsewhere.  Unlike the reference's GPU version, which uses
// expf and an online maximum, the probabilities here are the CPU reference's bits:
// carbon/src/cpu/kernels.cpp:799-828 (exp_neg, the sum in class order after the maximum).
#pragma once

#include <cstdint>

#include "dw_head.cuh"  // exp_neg_d

namespace crec {

// One block a line, a thread a frame: the reads run along the frames for each class.
// Writes arg[i][t] and, for a non-blank best, prob[i][t]; frames at or past the line's length
// and blank frames' probabilities are not written (the collapse reads neither).
__global__ void ctc_argmax_kernel(const float* logits, int classes, int frames, const int32_t* lengths, int32_t* arg,
                                  float* prob) {
  const int i = blockIdx.x;
  const int t_n = min(max(lengths[i], 0), frames);
  const float* line = logits + static_cast<size_t>(i) * classes * frames;
  for (int t = threadIdx.x; t < t_n; t += blockDim.x) {
    float best = -INFINITY;
    int a = 0;
    for (int c = 0; c < classes; ++c) {
      const float v = line[static_cast<size_t>(c) * frames + t];
      if (v > best) {
        best = v;
        a = c;
      }
    }
    arg[static_cast<size_t>(i) * frames + t] = a;
    if (a == 0) continue;
    float sum = 0.0f;
    for (int c = 0; c < classes; ++c) sum = __fadd_rn(sum, exp_neg_d(__fsub_rn(line[static_cast<size_t>(c) * frames + t], best)));
    prob[static_cast<size_t>(i) * frames + t] = __fdiv_rn(1.0f, sum);
  }
}

// carbon/src/lines.cpp:331-355 (ctc_collapse), a thread a line; line i's characters at
// [i * frames, i * frames + count[i]) of ids, starts and probs.
__global__ void ctc_collapse_lines_kernel(int n, int frames, const int32_t* lengths, const int32_t* arg,
                                          const float* prob, int32_t* ids, int32_t* starts, float* probs,
                                          int32_t* count) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int t_n = min(max(lengths[i], 0), frames);
  const size_t base = static_cast<size_t>(i) * frames;
  int prev = 0, k = 0;
  for (int t = 0; t < t_n; ++t) {
    const int id = arg[base + t];
    if (id != 0 && id != prev) {
      ids[base + k] = id;
      starts[base + k] = t;
      probs[base + k] = prob[base + t];
      ++k;
    } else if (id != 0) {
      const float p = prob[base + t], last = probs[base + k - 1];
      probs[base + k - 1] = last > p ? last : p;
    }
    prev = id;
  }
  count[i] = k;
}

}  // namespace crec
