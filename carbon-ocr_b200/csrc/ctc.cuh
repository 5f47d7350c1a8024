// Greedy CTC decoding of logits already in device memory: the unfused path
// (carbon::cuda::ctc_greedy, carbon/src/cuda/lines.cu:264-309 of the reference), for a
// recognizer whose last layer ran elsewhere.  Unlike the reference's GPU version, which uses
// expf and an online maximum, the probabilities here are the CPU reference's bits:
// carbon/src/cpu/kernels.cpp:799-828 (exp_neg, the sum in class order after the maximum).
#pragma once

#include <cstdint>

#include "crop_stem.cuh"  // dp4a_us
#include "dw_head.cuh"    // exp_neg_d

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

// The beam's candidates (carbon::PipelineModels::candidates, carbon/include/carbon/pipeline.h:133-141;
// the CPU's carbon/src/cpu/kernels.cpp:617-665, ctc_topk) of frames of the last run: a frame's logits
// made again from the head's input the run left in memory, then its best logit, the class-order
// sum of exp_neg(logit - best) and its topk likeliest classes but the blank (insertion in class
// order: a later class must beat a kept one, so ties keep the lower id).  The host finishes each
// frame with ln of the sum (the C library's logf, as the CPU reference takes it).
struct CandParams {
  const uint8_t* x;    // the head's input: column c's channels at x + c * cp * eb
  int cp, k, classes, topk;  // k: the input's channels padded (cp), a multiple of 16 bytes
  const int8_t* w8;    // INT8 [classes][k], zeros past the real channels
  const float* wf;     // FP16 [classes][k], the weights' float16 values, zeros past the real channels
  const int32_t* colsum;  // INT8 [classes]
  const float* scale;     // INT8 [classes] input scale x weight scale
  const float* bias;      // [classes]
  int in_zero, out_zero;
  float out_inv_scale;
  const float* table;  // INT8 [256]: a code's logit
  const int32_t* cols; // [frames] each frame's column
  int frames;
  int32_t* ids;        // [frames][topk]
  float* vals;         // [frames][topk] their logits
  float* best;         // [frames]
  float* sum;          // [frames]
  float* blank;        // [frames] the blank's logit
};

constexpr int kCandThreads = 256;

// One CTA a frame: the frame's channels into shared memory, a thread a class's logit (INT8: the
// head's integer sum and its output stage, operation by operation as the fused head does them, so
// the codes are the run's; FP16: an FP32 fma chain in channel order from 0, then + bias, within
// about 1e-3 of the tensor cores' sums), then one thread the frame's maximum, sum and top k.
template <bool kInt8>
__global__ void __launch_bounds__(kCandThreads) candidates_kernel(const __grid_constant__ CandParams p) {
  extern __shared__ __align__(16) uint8_t sm[];
  float* logit = reinterpret_cast<float*>(sm);                          // [classes]
  uint8_t* xs = sm + static_cast<size_t>(p.classes) * 4;                // [k * eb], 4-byte aligned (read a word at a time)
  const int f = blockIdx.x;
  const int eb = kInt8 ? 1 : 2;
  const uint8_t* src = p.x + static_cast<long long>(p.cols[f]) * p.cp * eb;
  for (int i = threadIdx.x; i < p.k * eb; i += blockDim.x) xs[i] = src[i];
  __syncthreads();
  for (int c = threadIdx.x; c < p.classes; c += blockDim.x) {
    if constexpr (kInt8) {
      const uint32_t* xw = reinterpret_cast<const uint32_t*>(xs);
      const int8_t* w = p.w8 + static_cast<size_t>(c) * p.k;
      int32_t acc = 0;
      for (int j = 0; j < p.k; j += 4) {
        const uint32_t wv = static_cast<uint32_t>(static_cast<uint8_t>(w[j])) |
                            static_cast<uint32_t>(static_cast<uint8_t>(w[j + 1])) << 8 |
                            static_cast<uint32_t>(static_cast<uint8_t>(w[j + 2])) << 16 |
                            static_cast<uint32_t>(static_cast<uint8_t>(w[j + 3])) << 24;
        acc = dp4a_us(xw[j >> 2], wv, acc);
      }
      const float v = __int2float_rn(acc - p.in_zero * p.colsum[c]);
      float q = __fmul_rn(__fadd_rn(__fmul_rn(v, p.scale[c]), p.bias[c]), p.out_inv_scale);
      q = fminf(fmaxf(q, static_cast<float>(-p.out_zero)), static_cast<float>(255 - p.out_zero));
      logit[c] = p.table[__float2int_rn(q) + p.out_zero];
    } else {
      const __half* xh = reinterpret_cast<const __half*>(xs);
      const float* w = p.wf + static_cast<size_t>(c) * p.k;
      float acc = 0.0f;
      for (int j = 0; j < p.k; ++j) acc = __fmaf_rn(w[j], __half2float(xh[j]), acc);
      logit[c] = __fadd_rn(acc, p.bias[c]);
    }
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  float best = -INFINITY;
  for (int c = 0; c < p.classes; ++c) best = logit[c] > best ? logit[c] : best;
  float sum = 0.0f;
  for (int c = 0; c < p.classes; ++c) sum = __fadd_rn(sum, exp_neg_d(__fsub_rn(logit[c], best)));
  float v[16];
  int32_t id[16];
  for (int q = 0; q < p.topk; ++q) {
    v[q] = -INFINITY;
    id[q] = 0;
  }
  if (p.topk > 0) {
    for (int c = 1; c < p.classes; ++c) {
      const float x = logit[c];
      if (!(x > v[p.topk - 1])) continue;
      int q = p.topk - 1;
      for (; q > 0 && v[q - 1] < x; --q) {
        v[q] = v[q - 1];
        id[q] = id[q - 1];
      }
      v[q] = x;
      id[q] = c;
    }
  }
  const size_t o = static_cast<size_t>(f) * p.topk;
  for (int q = 0; q < p.topk; ++q) {
    p.ids[o + q] = id[q];
    p.vals[o + q] = v[q];
  }
  p.best[f] = best;
  p.sum[f] = sum;
  p.blank[f] = logit[0];
}

}  // namespace crec
