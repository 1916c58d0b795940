// Native batch-1 greedy decode engine for the Qwen2.5 architecture, built
// around the b200 Linear kernels.
//
// It runs the same model as the reference engine (reference src/qwen2.cpp:
// embedding, per-layer RMSNorm -> QKV (+bias) -> RoPE -> GQA attention ->
// o_proj + residual -> RMSNorm -> gate/up -> SiLU*up -> down + residual,
// final RMSNorm, tied LM head with BF16 argmax), from the same qbin weights,
// but is organised for the GPU rather than for the host:
//   * q/k/v and gate/up weights are concatenated once at load, so a layer
//     has four Linear calls instead of seven;
//   * RMSNorm and SiLU*up are folded into the input staging of the decode
//     GEMV that consumes them, and the two residual adds into the epilogue
//     of the GEMV that produces them (GemvFusion, gemv.cu);
//   * the current token and position live in device memory: the LM-head
//     argmax kernel writes the next token, the position and the output
//     list, so a whole decode step -- 6 kernels per layer, 146 for the
//     24-layer model -- is one CUDA graph replayed without any host round
//     trip; the generated tokens are read back once at the end;
//   * kernels are launched with programmatic dependent launch, so each
//     GEMV's weight stream starts while the previous kernel finishes.
// Prefill runs the tensor-core GEMMs over all prompt tokens (M = prompt
// length) with row-wise RMSNorm / RoPE / causal attention kernels.
//
// The non-Linear kernels here are written for this engine; their
// arithmetic follows the reference's (FP32 math on BF16 values, BF16
// rounding at the same tensor boundaries; src/cuda/kernels.cu:18-324).
#include <cfloat>
#include <climits>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <new>
#include <vector>

#include "b200_engine.h"
#include "attention.cuh"
#include "common.cuh"
#include "kernels.h"
#include "persistent.h"

struct b200_engine {
  b200_engine_config cfg;
  std::vector<b200_engine_layer> layers;
  const uint16_t* embed = nullptr;
  const uint16_t* final_norm = nullptr;
  cudaStream_t stream = nullptr;
  int qkv_dim = 0;
  // device buffers (one allocation)
  void* arena = nullptr;
  b200::bf16 *x, *xn, *qkv, *att, *tmp, *gu, *h, *logits, *kcache, *vcache;
  float* lm_value;
  int* lm_index;
  int *d_token, *d_pos, *d_step, *d_out, *d_prompt;
  cudaGraphExec_t graph = nullptr;
  // persistent decode kernel (decode_persistent.cu)
  b200::PersistPlan plan;
  b200::PersistLayer* d_layers = nullptr;
  unsigned* grid_words = nullptr;  // [0] abort flag
  int* d_status = nullptr;
  unsigned long long* words = nullptr;  // tagged activations
  unsigned epoch = 0;                   // tags used so far
  int mode = B200_ENGINE_DECODE_GRAPH;
  int h_pos = -1;  // position of the next decode step (-1: no prefill yet)
  unsigned long long* trace = nullptr;  // persistent-kernel timeline (optional)
  int stall_phase = -1;                 // test hook for the next decode call
  int trace_count = 0;
};

namespace b200 {
namespace {

cudaLaunchConfig_t pdl_config(dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

// Rows of the embedding table for device-side token ids (16-byte copies).
__global__ void embed_kernel(const bf16* __restrict__ table, const int* __restrict__ tokens,
                             int hidden, bf16* __restrict__ out) {
  pdl_launch_dependents();
  pdl_wait_primary();
  const int t = blockIdx.x;
  const uint4* src = reinterpret_cast<const uint4*>(table + size_t(tokens[t]) * hidden);
  uint4* dst = reinterpret_cast<uint4*>(out + size_t(t) * hidden);
  for (int i = threadIdx.x; i < hidden / 8; i += blockDim.x) dst[i] = src[i];
}

// out[t] = bf16(x[t] * w * rsqrt(mean(x[t]^2) + eps)), one CTA per row.
__global__ void rmsnorm_rows_kernel(const bf16* __restrict__ in, const bf16* __restrict__ w,
                                    bf16* __restrict__ out, int hidden, float eps) {
  __shared__ float red[32];
  pdl_launch_dependents();
  pdl_wait_primary();
  const bf16* row = in + size_t(blockIdx.x) * hidden;
  float ss = 0.0f;
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
    const float v = __bfloat162float(row[i]);
    ss = fmaf(v, v, ss);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float total = 0.0f;
  for (int i = 0; i < int(blockDim.x >> 5); ++i) total += red[i];
  const float scale = rsqrtf(total / float(hidden) + eps);
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
    out[size_t(blockIdx.x) * hidden + i] = __float2bfloat16_rn(
        __bfloat162float(row[i]) * __bfloat162float(w[i]) * scale);
  }
}

// x = bf16(x + r), elementwise.
// x[row] = bf16(x[row] + r[row]), then out[row] = RMSNorm of the stored
// row (same roundings as add_kernel followed by rmsnorm_rows_kernel, one
// launch instead of two).
__global__ void add_rmsnorm_rows_kernel(bf16* __restrict__ x, const bf16* __restrict__ r,
                                        const bf16* __restrict__ w, bf16* __restrict__ out,
                                        int hidden, float eps) {
  __shared__ float red[32];
  pdl_launch_dependents();
  pdl_wait_primary();
  bf16* row = x + size_t(blockIdx.x) * hidden;
  const bf16* rrow = r + size_t(blockIdx.x) * hidden;
  float ss = 0.0f;
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
    const bf16 s = __float2bfloat16_rn(__bfloat162float(row[i]) + __bfloat162float(rrow[i]));
    row[i] = s;
    const float v = __bfloat162float(s);
    ss = fmaf(v, v, ss);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float total = 0.0f;
  for (int i = 0; i < int(blockDim.x >> 5); ++i) total += red[i];
  const float scale = rsqrtf(total / float(hidden) + eps);
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
    out[size_t(blockIdx.x) * hidden + i] = __float2bfloat16_rn(
        __bfloat162float(row[i]) * __bfloat162float(w[i]) * scale);
  }
}
__global__ void add_kernel(bf16* __restrict__ x, const bf16* __restrict__ r, size_t n) {
  pdl_launch_dependents();
  pdl_wait_primary();
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n;
       i += size_t(gridDim.x) * blockDim.x) {
    x[i] = __float2bfloat16_rn(__bfloat162float(x[i]) + __bfloat162float(r[i]));
  }
}

// h[t, i] = bf16(silu(g) * u) with [g | u] = gu[t].
__global__ void silu_mul_kernel(const bf16* __restrict__ gu, bf16* __restrict__ h, int t_rows,
                                int inter) {
  pdl_launch_dependents();
  pdl_wait_primary();
  const size_t n = size_t(t_rows) * inter;
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n;
       i += size_t(gridDim.x) * blockDim.x) {
    const size_t t = i / inter, c = i - t * inter;
    const float g = __bfloat162float(gu[t * 2 * inter + c]);
    const float u = __bfloat162float(gu[t * 2 * inter + inter + c]);
    h[i] = __float2bfloat16_rn(g / (1.0f + expf(-g)) * u);
  }
}

// Rotary embedding of q and k (half-split pairs (i, i + d/2), frequency
// theta^(-2i/d)) at position pos0 + t (or *d_pos), rotated q written back in
// place, rotated k and v stored to this layer's cache [kv_head][max_seq][d].
__global__ void rope_store_kernel(bf16* __restrict__ qkv, int qkv_dim, int heads, int kv_heads,
                                  int hd, float theta, int pos0, const int* __restrict__ d_pos,
                                  bf16* __restrict__ kcache, bf16* __restrict__ vcache,
                                  int max_seq) {
  pdl_launch_dependents();
  pdl_wait_primary();
  const int t = blockIdx.x;
  const int pos = (d_pos ? *d_pos : pos0) + t;
  const int half = hd / 2;
  bf16* row = qkv + size_t(t) * qkv_dim;
  const int pairs = (heads + kv_heads) * half;
  for (int j = threadIdx.x; j < pairs; j += blockDim.x) {
    const int head = j / half, i = j % half;
    const float freq = powf(theta, -2.0f * float(i) / float(hd));
    float sn, cs;
    sincosf(float(pos) * freq, &sn, &cs);
    bf16* v = row + head * hd;
    const float a = __bfloat162float(v[i]), b = __bfloat162float(v[i + half]);
    const bf16 ra = __float2bfloat16_rn(a * cs - b * sn);
    const bf16 rb = __float2bfloat16_rn(b * cs + a * sn);
    if (head < heads) {
      v[i] = ra;
      v[i + half] = rb;
    } else {
      const int kh = head - heads;
      bf16* kc = kcache + (size_t(kh) * max_seq + pos) * hd;
      kc[i] = ra;
      kc[i + half] = rb;
    }
  }
  const bf16* vsrc = row + (heads + kv_heads) * hd;
  for (int j = threadIdx.x; j < kv_heads * hd; j += blockDim.x) {
    const int kh = j / hd, d = j % hd;
    vcache[(size_t(kh) * max_seq + pos) * hd + d] = vsrc[j];
  }
}

// Causal GQA attention for query rows t at positions pos0 + t (or *d_pos),
// one CTA per (head, t) over the cache rows written by rope_store_kernel
// (attend_row, attention.cuh).
__global__ void __launch_bounds__(128)
attention_kernel(const bf16* __restrict__ qkv, int qkv_dim, const bf16* kcache,
                 const bf16* vcache, bf16* __restrict__ out, int heads,
                 int kv_heads, int hd, int max_seq, int pos0, const int* __restrict__ d_pos) {
  extern __shared__ float att_smem[];
  __shared__ float qs[kHeadDim];
  pdl_launch_dependents();
  pdl_wait_primary();
  const int head = blockIdx.x, t = blockIdx.y;
  const int seq = (d_pos ? *d_pos : pos0) + t + 1;
  const int kvh = head / (heads / kv_heads);
  const bf16* q = qkv + size_t(t) * qkv_dim + head * hd;
  if (threadIdx.x < kHeadDim) qs[threadIdx.x] = __bfloat162float(q[threadIdx.x]);
  __syncthreads();
  bf16* o = out + size_t(t) * heads * hd + head * hd;
  attend_row<128>(qs, kcache + size_t(kvh) * max_seq * hd, vcache + size_t(kvh) * max_seq * hd,
                  seq, -1, nullptr, nullptr, att_smem, threadIdx.x, [] { __syncthreads(); },
                  [o](int d, float v) { o[d] = __float2bfloat16_rn(v); });
}

// Final argmax of the LM head (lowest index on ties) feeding the next step:
// writes the token, appends it to the output list, advances step and
// position (set_pos >= 0 sets the position instead, after a prefill).
__global__ void __launch_bounds__(1024)
argmax_step_kernel(const float* __restrict__ bv, const int* __restrict__ bi, int count,
                   int* __restrict__ d_token, int* __restrict__ d_out, int* __restrict__ d_step,
                   int* __restrict__ d_pos, int set_pos, int max_out) {
  __shared__ float sv[32];
  __shared__ int si[32];
  pdl_launch_dependents();
  pdl_wait_primary();
  float best = -FLT_MAX;
  int best_index = INT_MAX;
  auto upd = [&](float v, int i) {
    if (v > best || (v == best && v > -FLT_MAX && i < best_index)) {
      best = v;
      best_index = i;
    }
  };
  for (int i = threadIdx.x; i < count; i += blockDim.x) upd(bv[i], bi[i]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, off);
    const int oi = __shfl_xor_sync(0xffffffffu, best_index, off);
    upd(ov, oi);
  }
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = best;
    si[threadIdx.x >> 5] = best_index;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    best = -FLT_MAX;
    best_index = INT_MAX;
    for (int w = 0; w < int(blockDim.x >> 5); ++w) upd(sv[w], si[w]);
    const int tok = best_index == INT_MAX ? 0 : best_index;
    *d_token = tok;
    int step = set_pos >= 0 ? 0 : *d_step;
    if (step < max_out) d_out[step] = tok;
    *d_step = step + 1;
    *d_pos = set_pos >= 0 ? set_pos : *d_pos + 1;
  }
}

int grid_for(size_t n) {
  size_t g = (n + 255) / 256;
  return int(g < 148 * 8 ? g : 148 * 8);
}

}  // namespace
}  // namespace b200

using b200::bf16;

namespace {
// Prefill attention on the tensor cores from this many prompt tokens
// (B200_ATTN_TC=1 / 0 forces it on / off).
constexpr int kAttentionTcMinTokens = 64;
bool use_attention_tc(int tokens) {
  const char* e = getenv("B200_ATTN_TC");
  if (e != nullptr) return strcmp(e, "1") == 0;
  return tokens >= kAttentionTcMinTokens;
}


int check(cudaError_t e) { return e == cudaSuccess ? B200_OK : int(e); }

#define ENGINE_TRY(expr)                 \
  do {                                   \
    const int rc_ = (expr);              \
    if (rc_ != B200_OK) return rc_;      \
  } while (0)

template <class K, class... A>
int launch(K kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t s, A... args) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = b200::pdl_config(grid, block, smem, s, attr);
  return check(cudaLaunchKernelEx(&cfg, kernel, args...));
}

// One transformer layer's Linear + small kernels.
//   decode (t_rows == 1 with d_pos): fused GEMVs;
//   prefill (t_rows >= 1, pos0 = 0): GEMMs + row kernels.
int layer_forward(b200_engine* e, int l, int t_rows, bool decode) {
  const auto& c = e->cfg;
  const auto& L = e->layers[l];
  const int H = c.hidden, I = c.intermediate, hd = H / c.heads;
  const size_t kv_layer = size_t(c.kv_heads) * c.max_seq * hd;
  bf16* kc = e->kcache + kv_layer * l;
  bf16* vc = e->vcache + kv_layer * l;
  cudaStream_t s = e->stream;
  const bool w8 = c.w8 != 0;
  auto B = [](const uint16_t* p) { return reinterpret_cast<const bf16*>(p); };
  const int* dpos = decode ? e->d_pos : nullptr;
  if (decode) {
    b200::GemvFusion f;
    f.in_mode = 1;
    f.norm_w = B(L.input_norm);
    f.eps = c.eps;
    ENGINE_TRY(check(b200::launch_gemv(w8, L.qkv_w, B(L.qkv_s), B(L.qkv_b), e->x, e->qkv,
                                       e->qkv_dim, H, nullptr, nullptr, s, nullptr, &f)));
  } else {
    // Layers after the first receive xn = RMSNorm(x) from the previous
    // layer's fused residual add.
    if (l == 0) {
      ENGINE_TRY(launch(b200::rmsnorm_rows_kernel, dim3(t_rows), dim3(256), 0, s,
                        (const bf16*)e->x, B(L.input_norm), e->xn, H, c.eps));
    }
    ENGINE_TRY(w8 ? b200_gemm_w8a16(static_cast<const int8_t*>(L.qkv_w), L.qkv_s, 64, L.qkv_b,
                                    reinterpret_cast<const uint16_t*>(e->xn),
                                    reinterpret_cast<uint16_t*>(e->qkv), t_rows, e->qkv_dim, H, s)
                  : b200_gemm_bf16(static_cast<const uint16_t*>(L.qkv_w), L.qkv_b,
                                   reinterpret_cast<const uint16_t*>(e->xn),
                                   reinterpret_cast<uint16_t*>(e->qkv), t_rows, e->qkv_dim, H, s));
  }
  ENGINE_TRY(launch(b200::rope_store_kernel, dim3(t_rows), dim3(256), 0, s, e->qkv, e->qkv_dim,
                    c.heads, c.kv_heads, hd, c.theta, 0, dpos, kc, vc, c.max_seq));
  if (!decode && use_attention_tc(t_rows)) {
    ENGINE_TRY(check(b200::launch_attention_prefill_tc(
        (const bf16*)e->qkv, e->qkv_dim, (const bf16*)kc, (const bf16*)vc, e->att,
        c.heads * hd, t_rows, 0, c.heads, c.kv_heads, c.max_seq, s)));
  } else {
    ENGINE_TRY(launch(b200::attention_kernel, dim3(c.heads, t_rows), dim3(128),
                      b200::attend_smem_floats<128>(c.max_seq) * sizeof(float), s,
                      (const bf16*)e->qkv, e->qkv_dim,
                      (const bf16*)kc, (const bf16*)vc, e->att, c.heads, c.kv_heads, hd,
                      c.max_seq, 0, dpos));
  }
  if (decode) {
    b200::GemvFusion f;
    f.residual = e->x;
    ENGINE_TRY(check(b200::launch_gemv(w8, L.o_w, B(L.o_s), nullptr, e->att, e->tmp, H, H,
                                       nullptr, nullptr, s, nullptr, &f)));
    b200::GemvFusion g;
    g.in_mode = 1;
    g.norm_w = B(L.post_norm);
    g.eps = c.eps;
    ENGINE_TRY(check(b200::launch_gemv(w8, L.gate_up_w, B(L.gate_up_s), nullptr, e->x, e->gu,
                                       2 * I, H, nullptr, nullptr, s, nullptr, &g)));
    b200::GemvFusion d;
    d.in_mode = 2;
    d.residual = e->x;
    ENGINE_TRY(check(b200::launch_gemv(w8, L.down_w, B(L.down_s), nullptr, e->gu, e->tmp, H, I,
                                       nullptr, nullptr, s, nullptr, &d)));
    return B200_OK;
  }
  auto gemm = [&](const void* w, const uint16_t* sc, const bf16* in, bf16* out, int n, int k) {
    return w8 ? b200_gemm_w8a16(static_cast<const int8_t*>(w), sc, 64, nullptr,
                                reinterpret_cast<const uint16_t*>(in),
                                reinterpret_cast<uint16_t*>(out), t_rows, n, k, s)
              : b200_gemm_bf16(static_cast<const uint16_t*>(w), nullptr,
                               reinterpret_cast<const uint16_t*>(in),
                               reinterpret_cast<uint16_t*>(out), t_rows, n, k, s);
  };
  const size_t th = size_t(t_rows) * H;
  ENGINE_TRY(gemm(L.o_w, L.o_s, e->att, e->tmp, H, H));
  ENGINE_TRY(launch(b200::add_rmsnorm_rows_kernel, dim3(t_rows), dim3(256), 0, s, e->x,
                    (const bf16*)e->tmp, B(L.post_norm), e->xn, H, c.eps));
  ENGINE_TRY(gemm(L.gate_up_w, L.gate_up_s, e->xn, e->gu, 2 * I, H));
  ENGINE_TRY(launch(b200::silu_mul_kernel, dim3(b200::grid_for(size_t(t_rows) * I)), dim3(256),
                    0, s, (const bf16*)e->gu, e->h, t_rows, I));
  ENGINE_TRY(gemm(L.down_w, L.down_s, e->h, e->tmp, H, I));
  if (l + 1 < c.layers) {
    // Residual add fused with the next layer's input RMSNorm.
    ENGINE_TRY(launch(b200::add_rmsnorm_rows_kernel, dim3(t_rows), dim3(256), 0, s, e->x,
                      (const bf16*)e->tmp, B(e->layers[l + 1].input_norm), e->xn, H, c.eps));
  } else {
    ENGINE_TRY(launch(b200::add_kernel, dim3(b200::grid_for(th)), dim3(256), 0, s, e->x,
                      (const bf16*)e->tmp, th));
  }
  return B200_OK;
}

// Final RMSNorm (fused) + tied LM head on residual row `row`, then the
// argmax step kernel.
int head_forward(b200_engine* e, int row, int set_pos, int max_out) {
  const auto& c = e->cfg;
  b200::GemvFusion f;
  f.in_mode = 1;
  f.norm_w = reinterpret_cast<const bf16*>(e->final_norm);
  f.eps = c.eps;
  int grid = 0;
  ENGINE_TRY(check(b200::launch_gemv(false, e->embed, nullptr, nullptr,
                                     e->x + size_t(row) * c.hidden, e->logits, c.vocab, c.hidden,
                                     e->lm_value, e->lm_index, e->stream, &grid, &f)));
  return launch(b200::argmax_step_kernel, dim3(1), dim3(1024), 0, e->stream,
                (const float*)e->lm_value, (const int*)e->lm_index, grid, e->d_token, e->d_out,
                e->d_step, e->d_pos, set_pos, max_out);
}

int decode_step(b200_engine* e, int max_out) {
  const auto& c = e->cfg;
  ENGINE_TRY(launch(b200::embed_kernel, dim3(1), dim3(128), 0, e->stream,
                    reinterpret_cast<const bf16*>(e->embed), (const int*)e->d_token, c.hidden,
                    e->x));
  for (int l = 0; l < c.layers; ++l) ENGINE_TRY(layer_forward(e, l, 1, true));
  return head_forward(e, 0, -1, max_out);
}

}  // namespace

extern "C" {

int b200_engine_create(b200_engine_t* out, const b200_engine_config* cfg,
                       const b200_engine_layer* layers, const uint16_t* embed,
                       const uint16_t* final_norm, b200_stream_t stream) {
  if (out == nullptr || cfg == nullptr || layers == nullptr || embed == nullptr ||
      final_norm == nullptr) {
    return B200_ERR_INVALID_ARGUMENT;
  }
  const b200_engine_config& c = *cfg;
  if (c.hidden <= 0 || c.heads <= 0 || c.kv_heads <= 0 || c.hidden % c.heads != 0 ||
      c.heads % c.kv_heads != 0 || c.layers <= 0 || c.vocab <= 0 || c.max_seq <= 0 ||
      c.intermediate <= 0) {
    return B200_ERR_INVALID_ARGUMENT;
  }
  const int hd = c.hidden / c.heads;
  // Shapes the fused TMA-bulk GEMVs and the kernels above take.
  if (hd != 64 || c.hidden % 64 != 0 || c.intermediate % 64 != 0 || c.vocab % 8 != 0 ||
      c.max_seq > 8192) {
    return B200_ERR_TOO_LARGE;
  }
  // W8A16 prefill GEMMs dequantise the weights once into a library buffer:
  // reserved here, with the engine's own buffers (GEMM calls never allocate).
  if (c.w8 != 0) {
    const cudaError_t re = b200::reserve_gemm_scratch(0);
    if (re != cudaSuccess) return int(re);
  }
  auto* e = new (std::nothrow) b200_engine;
  if (e == nullptr) return B200_ERR_INVALID_ARGUMENT;
  e->cfg = c;
  e->layers.assign(layers, layers + c.layers);
  e->embed = embed;
  e->final_norm = final_norm;
  e->stream = stream;
  e->qkv_dim = (c.heads + 2 * c.kv_heads) * hd;
  const size_t T = c.max_seq, H = c.hidden, I = c.intermediate, V = c.vocab;
  const size_t kv = size_t(c.layers) * c.kv_heads * c.max_seq * hd;
  const size_t blocks = (V + 7) / 8;
  // Buffer sizes in bytes, each rounded to 256.
  const size_t sizes[] = {T * H * 2, T * H * 2, T * e->qkv_dim * 2, T * H * 2, T * H * 2,
                          T * 2 * I * 2, T * I * 2, V * 2, kv * 2, kv * 2, blocks * 4,
                          blocks * 4, 64, 64, 64, T * 4 + 64, T * 4 + 64,
                          size_t(c.layers) * sizeof(b200::PersistLayer), 64, 64};
  size_t total = 0;
  for (size_t sz : sizes) total += (sz + 255) / 256 * 256;
  cudaError_t err = cudaMalloc(&e->arena, total);
  if (err != cudaSuccess) {
    delete e;
    return int(err);
  }
  unsigned char* p = static_cast<unsigned char*>(e->arena);
  size_t i = 0;
  auto take = [&]() {
    void* r = p;
    p += (sizes[i++] + 255) / 256 * 256;
    return r;
  };
  e->x = static_cast<bf16*>(take());
  e->xn = static_cast<bf16*>(take());
  e->qkv = static_cast<bf16*>(take());
  e->att = static_cast<bf16*>(take());
  e->tmp = static_cast<bf16*>(take());
  e->gu = static_cast<bf16*>(take());
  e->h = static_cast<bf16*>(take());
  e->logits = static_cast<bf16*>(take());
  e->kcache = static_cast<bf16*>(take());
  e->vcache = static_cast<bf16*>(take());
  e->lm_value = static_cast<float*>(take());
  e->lm_index = static_cast<int*>(take());
  e->d_token = static_cast<int*>(take());
  e->d_pos = static_cast<int*>(take());
  e->d_step = static_cast<int*>(take());
  e->d_out = static_cast<int*>(take());
  e->d_prompt = static_cast<int*>(take());
  e->d_layers = static_cast<b200::PersistLayer*>(take());
  e->grid_words = static_cast<unsigned*>(take());
  e->d_status = static_cast<int*>(take());
  std::vector<b200::PersistLayer> pl(c.layers);
  for (int l = 0; l < c.layers; ++l) {
    const b200_engine_layer& L = layers[l];
    auto B = [](const uint16_t* q) { return reinterpret_cast<const bf16*>(q); };
    pl[l] = {L.qkv_w, B(L.qkv_s), B(L.qkv_b), L.o_w, B(L.o_s), L.gate_up_w, B(L.gate_up_s),
             L.down_w, B(L.down_s), B(L.input_norm), B(L.post_norm)};
  }
  err = cudaMemcpy(e->d_layers, pl.data(), pl.size() * sizeof(b200::PersistLayer),
                   cudaMemcpyHostToDevice);
  if (err == cudaSuccess) err = cudaMemset(e->d_status, 0, sizeof(int));
  if (err != cudaSuccess) {
    cudaFree(e->arena);
    delete e;
    return int(err);
  }
  e->plan = b200::plan_persistent(c.w8 != 0, c.hidden, c.intermediate, c.heads, c.kv_heads,
                                  c.vocab, c.max_seq);
  if (e->plan.ok) {
    const size_t bytes = b200::persist_words(c.layers, e->qkv_dim, c.hidden, c.intermediate,
                                             e->plan.grid) * sizeof(unsigned long long);
    err = cudaMalloc(&e->words, bytes);
    if (err == cudaSuccess) err = cudaMemset(e->words, 0, bytes);
    if (err != cudaSuccess) {
      cudaGetLastError();
      if (e->words) cudaFree(e->words);
      e->words = nullptr;
      e->plan.ok = false;
    }
  }
  e->mode = e->plan.ok ? B200_ENGINE_DECODE_PERSISTENT : B200_ENGINE_DECODE_GRAPH;
  *out = e;
  return B200_OK;
}

int b200_engine_destroy(b200_engine_t e) {
  if (e == nullptr) return B200_OK;
  if (e->graph) cudaGraphExecDestroy(e->graph);
  if (e->trace) cudaFree(e->trace);
  if (e->words) cudaFree(e->words);
  cudaFree(e->arena);
  delete e;
  return B200_OK;
}

int b200_engine_prefill(b200_engine_t e, const int* prompt, int n) {
  if (e == nullptr || prompt == nullptr || n <= 0 || n > e->cfg.max_seq) {
    return B200_ERR_INVALID_ARGUMENT;
  }
  ENGINE_TRY(check(cudaMemcpyAsync(e->d_prompt, prompt, size_t(n) * sizeof(int),
                                   cudaMemcpyHostToDevice, e->stream)));
  ENGINE_TRY(launch(b200::embed_kernel, dim3(n), dim3(128), 0, e->stream,
                    reinterpret_cast<const bf16*>(e->embed), (const int*)e->d_prompt,
                    e->cfg.hidden, e->x));
  for (int l = 0; l < e->cfg.layers; ++l) ENGINE_TRY(layer_forward(e, l, n, false));
  ENGINE_TRY(head_forward(e, n - 1, n, e->cfg.max_seq));
  e->h_pos = n;
  return B200_OK;
}

int b200_engine_set_decode_mode(b200_engine_t e, int mode) {
  if (e == nullptr) return B200_ERR_INVALID_ARGUMENT;
  if (mode == B200_ENGINE_DECODE_GRAPH) {
    e->mode = mode;
    return B200_OK;
  }
  if (mode != B200_ENGINE_DECODE_PERSISTENT) return B200_ERR_INVALID_ARGUMENT;
  if (!e->plan.ok) return B200_ERR_TOO_LARGE;
  e->mode = mode;
  return B200_OK;
}

int b200_engine_set_trace(b200_engine_t e, int phases) {
  if (e == nullptr || phases < 0) return B200_ERR_INVALID_ARGUMENT;
  if (e->trace) {
    ENGINE_TRY(check(cudaStreamSynchronize(e->stream)));
    cudaFree(e->trace);
    e->trace = nullptr;
    e->trace_count = 0;
  }
  if (phases == 0) return B200_OK;
  if (!e->plan.ok) return B200_ERR_TOO_LARGE;
  const size_t bytes = size_t(e->plan.grid) * phases * 4 * sizeof(unsigned long long);
  ENGINE_TRY(check(cudaMalloc(&e->trace, bytes)));
  ENGINE_TRY(check(cudaMemset(e->trace, 0, bytes)));
  e->trace_count = phases;
  return B200_OK;
}

int b200_engine_read_trace(b200_engine_t e, unsigned long long* out) {
  if (e == nullptr) return B200_ERR_INVALID_ARGUMENT;
  if (e->trace == nullptr) return 0;
  if (out != nullptr) {
    const size_t n = size_t(e->plan.grid) * e->trace_count * 4;
    ENGINE_TRY(check(cudaMemcpyAsync(out, e->trace, n * sizeof(unsigned long long),
                                     cudaMemcpyDeviceToHost, e->stream)));
    ENGINE_TRY(check(cudaStreamSynchronize(e->stream)));
  }
  return e->plan.grid;
}

int b200_engine_test_stall(b200_engine_t e, int phase) {
  if (e == nullptr) return B200_ERR_INVALID_ARGUMENT;
  if (e->mode != B200_ENGINE_DECODE_PERSISTENT) return B200_ERR_INVALID_ARGUMENT;
  e->stall_phase = phase < 0 ? -1 : phase;
  return B200_OK;
}

int b200_engine_decode_mode(b200_engine_t e) {
  return e == nullptr ? B200_ERR_INVALID_ARGUMENT : e->mode;
}

int b200_engine_device_status(b200_engine_t e, int clear) {
  if (e == nullptr) return B200_ERR_INVALID_ARGUMENT;
  int v = 0;
  cudaError_t err = cudaMemcpyAsync(&v, e->d_status, sizeof(int), cudaMemcpyDeviceToHost,
                                    e->stream);
  if (err == cudaSuccess) err = cudaStreamSynchronize(e->stream);
  if (err == cudaSuccess && clear) err = cudaMemset(e->d_status, 0, sizeof(int));
  if (err != cudaSuccess) return -int(err);
  return v;
}

int b200_engine_decode(b200_engine_t e, int steps) {
  if (e == nullptr || steps < 0) return B200_ERR_INVALID_ARGUMENT;
  if (steps == 0) return B200_OK;
  // Each step writes the KV cache at its position: the prompt plus the
  // decoded tokens must fit max_seq.
  if (e->h_pos < 0) return B200_ERR_INVALID_ARGUMENT;
  if (steps > e->cfg.max_seq - e->h_pos) return B200_ERR_TOO_LARGE;
  // h_pos mirrors the device position: it advances only by the steps whose
  // launches were accepted, so a failed launch leaves it consistent.
  if (e->mode == B200_ENGINE_DECODE_PERSISTENT) {
    const auto& c = e->cfg;
    b200::PersistArgs a = {};
    a.layers = e->d_layers;
    a.n_layers = c.layers;
    a.hidden = c.hidden;
    a.inter = c.intermediate;
    a.heads = c.heads;
    a.kv_heads = c.kv_heads;
    a.vocab = c.vocab;
    a.max_seq = c.max_seq;
    a.eps = c.eps;
    a.theta = c.theta;
    a.embed = reinterpret_cast<const bf16*>(e->embed);
    a.final_norm = reinterpret_cast<const bf16*>(e->final_norm);
    a.words = e->words;
    a.epoch = e->epoch;
    a.logits = e->logits;
    a.kcache = e->kcache;
    a.vcache = e->vcache;
    a.d_token = e->d_token;
    a.d_pos = e->d_pos;
    a.d_step = e->d_step;
    a.d_out = e->d_out;
    a.max_out = c.max_seq;
    a.grid_abort = reinterpret_cast<int*>(e->grid_words);
    a.status = e->d_status;
    a.trace = e->trace;
    a.trace_count = e->trace_count;
    a.stall_phase = e->stall_phase;
    e->stall_phase = -1;
    a.steps = steps;
    const int rc = check(b200::launch_persistent(c.w8 != 0, e->plan, a, e->stream));
    if (rc != B200_OK) return rc;
    e->epoch += unsigned(steps);
    e->h_pos += steps;
    return B200_OK;
  }
  if (e->graph == nullptr) {
    cudaGraph_t g = nullptr;
    ENGINE_TRY(check(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal)));
    const int rc = decode_step(e, e->cfg.max_seq);
    const cudaError_t end = cudaStreamEndCapture(e->stream, &g);
    if (rc != B200_OK) return rc;
    ENGINE_TRY(check(end));
    const cudaError_t inst = cudaGraphInstantiate(&e->graph, g, 0);
    cudaGraphDestroy(g);
    ENGINE_TRY(check(inst));
  }
  for (int i = 0; i < steps; ++i) {
    ENGINE_TRY(check(cudaGraphLaunch(e->graph, e->stream)));
    e->h_pos += 1;
  }
  return B200_OK;
}

int b200_attention_prefill_bf16(const uint16_t* q, int q_stride, const uint16_t* kcache,
                                const uint16_t* vcache, uint16_t* out, int out_stride,
                                int tokens, int pos0, int heads, int kv_heads, int max_seq,
                                b200_stream_t stream) {
  if (q == nullptr || kcache == nullptr || vcache == nullptr || out == nullptr || tokens < 0 ||
      pos0 < 0 || heads <= 0 || kv_heads <= 0 || heads % kv_heads != 0 ||
      q_stride < heads * 64 || out_stride < heads * 64 || q_stride % 8 != 0 ||
      out_stride % 8 != 0 || pos0 + tokens > max_seq) {
    return B200_ERR_INVALID_ARGUMENT;
  }
  if (tokens == 0) return B200_OK;
  return check(b200::launch_attention_prefill_tc(
      reinterpret_cast<const bf16*>(q), q_stride, reinterpret_cast<const bf16*>(kcache),
      reinterpret_cast<const bf16*>(vcache), reinterpret_cast<bf16*>(out), out_stride, tokens,
      pos0, heads, kv_heads, max_seq, reinterpret_cast<cudaStream_t>(stream)));
}

int b200_engine_force_token(b200_engine_t e, int token) {
  if (e == nullptr || token < 0 || token >= e->cfg.vocab) return B200_ERR_INVALID_ARGUMENT;
  if (e->h_pos < 0) return B200_ERR_INVALID_ARGUMENT;
  return check(cudaMemcpyAsync(e->d_token, &token, sizeof(int), cudaMemcpyHostToDevice,
                               e->stream));
}

int b200_engine_tokens(b200_engine_t e, int* out, int count) {
  if (e == nullptr || out == nullptr || count < 0 || count > e->cfg.max_seq) {
    return B200_ERR_INVALID_ARGUMENT;
  }
  ENGINE_TRY(check(cudaMemcpyAsync(out, e->d_out, size_t(count) * sizeof(int),
                                   cudaMemcpyDeviceToHost, e->stream)));
  return check(cudaStreamSynchronize(e->stream));
}

int b200_engine_logits(b200_engine_t e, uint16_t* out) {
  if (e == nullptr || out == nullptr) return B200_ERR_INVALID_ARGUMENT;
  ENGINE_TRY(check(cudaMemcpyAsync(out, e->logits, size_t(e->cfg.vocab) * 2,
                                   cudaMemcpyDeviceToHost, e->stream)));
  return check(cudaStreamSynchronize(e->stream));
}

}  // extern "C"
