/*
 * CPU restatement of the reference's Linear-layer arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker that the CUDA kernels
 * are compared against; it is never linked into the product library and no
 * product code path calls it.  Only tests/, __graft_entry__.smoke() and the
 * CPU-baseline leg of bench.py load it.
 *
 * Every function names the reference file:line whose behaviour it restates
 * (paths are relative to the reference project root).  Results are written
 * as IEEE fp32 or as BF16 bit patterns (uint16_t) so Python can compare them
 * bit for bit.  Each output element is computed sequentially over k, in the
 * order the reference's CPU restatements use, so the result does not depend
 * on how many OpenMP threads run the outer loops.
 *
 * Build: see oracle/Makefile (gcc -O2 -ffp-contract=off -fopenmp).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

/* BF16 round-to-nearest-even, NaN kept quiet.
 * tests/test_cuda.cpp:16-22 (float_to_bf16) and
 * tools/export_model.py:123-131 (float32_to_bfloat16, including NaN rule). */
uint16_t oracle_f32_to_bf16(float value) {
  uint32_t bits;
  memcpy(&bits, &value, sizeof(bits));
  if ((bits & 0x7f800000u) == 0x7f800000u && (bits & 0x007fffffu) != 0u) {
    return (uint16_t)((bits >> 16) | 0x0040u);
  }
  const uint32_t round = 0x7fffu + ((bits >> 16) & 1u);
  return (uint16_t)((bits + round) >> 16);
}

/* tests/test_cuda.cpp:24-28 (bf16_to_float). */
float oracle_bf16_to_f32(uint16_t value) {
  const uint32_t bits = (uint32_t)value << 16;
  float result;
  memcpy(&result, &bits, sizeof(result));
  return result;
}

void oracle_f32_to_bf16_array(const float* in, uint16_t* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = oracle_f32_to_bf16(in[i]);
}

void oracle_bf16_to_f32_array(const uint16_t* in, float* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = oracle_bf16_to_f32(in[i]);
}

/* BF16 Linear, FP32 result (not rounded): sum starts at the bias and adds
 * w*x in k order.  tests/test_cuda.cpp:474-490 (linear_reference). */
void oracle_linear_bf16(const uint16_t* weight, const uint16_t* bias,
                        const uint16_t* input, float* output, int tokens,
                        int out_features, int in_features) {
#pragma omp parallel for collapse(2) schedule(static)
  for (int t = 0; t < tokens; ++t) {
    for (int n = 0; n < out_features; ++n) {
      const uint16_t* w = weight + (int64_t)n * in_features;
      const uint16_t* x = input + (int64_t)t * in_features;
      float sum = bias ? oracle_bf16_to_f32(bias[n]) : 0.0f;
      for (int k = 0; k < in_features; ++k) {
        sum += oracle_bf16_to_f32(w[k]) * oracle_bf16_to_f32(x[k]);
      }
      output[(int64_t)t * out_features + n] = sum;
    }
  }
}

/* W8A16 Linear.  dequant_mode 0: the GEMV arithmetic, dequantised weight is
 * float(q) * scale in FP32 (tests/test_cuda.cpp:492-517 w8a16_reference;
 * src/cuda/kernels.cu:953-983 dot_w8a16_sixteen).  dequant_mode 1: the
 * tensor-core GEMM arithmetic, where the dequantised weight is first rounded
 * to BF16 (src/cuda/kernels.cu:1075-1094 dequant_w8a16_stage).  Accumulate
 * with fmaf in k order, add bias after the sum, round to BF16.  Scales are
 * [out_features, ceil(in_features / group_size)] BF16. */
void oracle_linear_w8a16(const int8_t* weight, const uint16_t* scales,
                         int group_size, const uint16_t* bias,
                         const uint16_t* input, uint16_t* output, int tokens,
                         int out_features, int in_features,
                         int dequant_mode) {
  const int groups = (in_features + group_size - 1) / group_size;
#pragma omp parallel for collapse(2) schedule(static)
  for (int t = 0; t < tokens; ++t) {
    for (int n = 0; n < out_features; ++n) {
      const int8_t* w = weight + (int64_t)n * in_features;
      const uint16_t* s = scales + (int64_t)n * groups;
      const uint16_t* x = input + (int64_t)t * in_features;
      float sum = 0.0f;
      for (int k = 0; k < in_features; ++k) {
        float dq = (float)w[k] * oracle_bf16_to_f32(s[k / group_size]);
        if (dequant_mode == 1) dq = oracle_bf16_to_f32(oracle_f32_to_bf16(dq));
        sum = fmaf(dq, oracle_bf16_to_f32(x[k]), sum);
      }
      if (bias) sum += oracle_bf16_to_f32(bias[n]);
      output[(int64_t)t * out_features + n] = oracle_f32_to_bf16(sum);
    }
  }
}

/* Argmax over BF16 values, lowest index on ties.  Restates
 * src/cuda/kernels.cu:326-356 (argmax_bf16_kernel): the running best starts
 * at -FLT_MAX with index 0 and only a strictly greater value replaces it, so
 * NaN, -inf and -FLT_MAX never win and an input with no value above -FLT_MAX
 * (or n <= 0) yields index 0.  The host check of tests/test_cuda.cpp:853-867
 * agrees on every finite input. */
int oracle_argmax_bf16(const uint16_t* values, int n) {
  int best_index = 0;
  float best = -3.40282347e+38f;
  for (int i = 0; i < n; ++i) {
    const float v = oracle_bf16_to_f32(values[i]);
    if (v > best) {
      best = v;
      best_index = i;
    }
  }
  return best_index;
}

/* Fused LM head: logits = bf16(sum + bias) with the reference's per-row sum,
 * then argmax over the BF16-rounded logits, lowest index on ties.
 * src/cuda/kernels.cu:492-603 (lm_head_bf16_kernel + lm_head_reduce_kernel).
 * weight_int8 != 0 selects the W8A16 form (GEMV dequant arithmetic) used for
 * the synthetic 896->151936 W8 shape, which has no reference kernel: it is
 * gemv_w8a16 (src/cuda/kernels.cu:1627-1655) followed by argmax_bf16. */
int oracle_lm_head(const void* weight, const uint16_t* scales, int group_size,
                   const uint16_t* bias, const uint16_t* input,
                   uint16_t* logits, int vocab, int in_features,
                   int weight_int8) {
  if (weight_int8) {
    oracle_linear_w8a16((const int8_t*)weight, scales, group_size, bias, input,
                        logits, 1, vocab, in_features, 0);
  } else {
    const uint16_t* w = (const uint16_t*)weight;
#pragma omp parallel for schedule(static)
    for (int n = 0; n < vocab; ++n) {
      float sum = 0.0f;
      for (int k = 0; k < in_features; ++k) {
        sum = fmaf(oracle_bf16_to_f32(w[(int64_t)n * in_features + k]),
                   oracle_bf16_to_f32(input[k]), sum);
      }
      if (bias) sum += oracle_bf16_to_f32(bias[n]);
      logits[n] = oracle_f32_to_bf16(sum);
    }
  }
  return oracle_argmax_bf16(logits, vocab);
}

/* Symmetric group-wise INT8 quantiser, group along K.
 * tools/export_model.py:226-247 (quantize_groupwise) and :289-296:
 *   scale = max|w| / 127 per (row, group) in FP32, 0 -> 1.0;
 *   q = clip(rint(w / scale), -127, 127), rint = round-half-even;
 *   stored scale = bf16_rne(scale) (the q values use the FP32 scale). */
void oracle_quantize_groupwise(const float* weight, int rows, int columns,
                               int group_size, int8_t* q_out,
                               uint16_t* scale_out) {
  const int groups = (columns + group_size - 1) / group_size;
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; ++r) {
    const float* w = weight + (int64_t)r * columns;
    for (int g = 0; g < groups; ++g) {
      const int begin = g * group_size;
      const int end = begin + group_size < columns ? begin + group_size : columns;
      float amax = 0.0f;
      for (int c = begin; c < end; ++c) {
        const float a = fabsf(w[c]);
        if (a > amax) amax = a;
      }
      float scale = amax / 127.0f;
      if (scale == 0.0f) scale = 1.0f;
      for (int c = begin; c < end; ++c) {
        float v = nearbyintf(w[c] / scale);
        if (v < -127.0f) v = -127.0f;
        if (v > 127.0f) v = 127.0f;
        q_out[(int64_t)r * columns + c] = (int8_t)v;
      }
      scale_out[(int64_t)r * groups + g] = oracle_f32_to_bf16(scale);
    }
  }
}

/* Decode GEMV / LM-head logits in the reference CUDA kernels' exact FP32
 * operation order (bit-exact restatement of their arithmetic; denormals are
 * not flushed here, which the reference's --use_fast_math build does; no
 * realistic Linear produces them).  Returns BF16 bits in `out`.
 *   w8 = 1: gemv_w8a16_fast_kernel (src/cuda/kernels.cu:953-1041, 1627-1655):
 *     16-element chunks; chunk dot d = fma(q0*s, x0, 0), d = fma(q_i*s, x_i, d).
 *   w8 = 0: gemv_bf16_fast_kernel / lm_head_bf16_kernel (kernels.cu:359-384,
 *     438-490, 492-568): 8-element chunks (dot_bf16_eight:
 *     d = fma(w0, x0, w1*x1); d = fma(w2j, x2j, fma(w2j+1, x2j+1, d))).
 *   Lane l of warp slice ws (of W warps per row) adds chunks
 *   l + 32*ws + 32*W*j to a sum starting at 0; the 32 lane sums meet in the
 *   __shfl_down tree (lane i += lane i+off, off = 16..1); W > 1 partials are
 *   added in warp order to 0; then + bias, BF16 RNE.
 *   W = 4 when in_features > 1024 for a GEMV (kernels.cu:1547-1558,
 *   1636-1651), W = 1 otherwise and always for the BF16 LM head. */
void oracle_gemv_reference_order(const void* weight, int w8, const uint16_t* scales,
                                 const uint16_t* bias, const uint16_t* input,
                                 uint16_t* out, int n_rows, int k, int lm_head) {
  const int epc = w8 ? 16 : 8;
  const int chunks = k / epc;
  const int groups = k / 64;
  const int wpr = (k > 1024 && (w8 || !lm_head)) ? 4 : 1;
#pragma omp parallel for schedule(static)
  for (int r = 0; r < n_rows; ++r) {
    float partial[4];
    for (int ws = 0; ws < wpr; ++ws) {
      float lane_sum[32];
      for (int l = 0; l < 32; ++l) {
        float sum = 0.0f;
        for (int c = l + 32 * ws; c < chunks; c += 32 * wpr) {
          float d;
          if (w8) {
            const int8_t* q = (const int8_t*)weight + (int64_t)r * k + c * 16;
            const float s = oracle_bf16_to_f32(scales[(int64_t)r * groups + c / 4]);
            const uint16_t* x = input + c * 16;
            d = fmaf((float)q[0] * s, oracle_bf16_to_f32(x[0]), 0.0f);
            for (int e = 1; e < 16; ++e) {
              d = fmaf((float)q[e] * s, oracle_bf16_to_f32(x[e]), d);
            }
          } else {
            const uint16_t* w = (const uint16_t*)weight + (int64_t)r * k + c * 8;
            const uint16_t* x = input + c * 8;
#define WF(i) oracle_bf16_to_f32(w[i])
#define XF(i) oracle_bf16_to_f32(x[i])
            d = fmaf(WF(0), XF(0), WF(1) * XF(1));
            d = fmaf(WF(2), XF(2), fmaf(WF(3), XF(3), d));
            d = fmaf(WF(4), XF(4), fmaf(WF(5), XF(5), d));
            d = fmaf(WF(6), XF(6), fmaf(WF(7), XF(7), d));
#undef WF
#undef XF
          }
          sum += d;
        }
        lane_sum[l] = sum;
      }
      for (int off = 16; off > 0; off >>= 1) {
        for (int i = 0; i < off; ++i) lane_sum[i] = lane_sum[i] + lane_sum[i + off];
      }
      partial[ws] = lane_sum[0];
    }
    float total;
    if (wpr > 1) {
      total = 0.0f;
      for (int ws = 0; ws < wpr; ++ws) total += partial[ws];
    } else {
      total = partial[0];
    }
    const float b = bias ? oracle_bf16_to_f32(bias[r]) : 0.0f;
    out[r] = oracle_f32_to_bf16(total + b);
  }
}
