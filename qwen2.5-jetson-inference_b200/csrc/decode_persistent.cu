// Persistent decode kernel: every greedy decode step of the Qwen2.5 model
// (all layers, the LM head and the argmax) in one cooperative launch, one
// CTA per SM, for any number of steps.
//
// A decode step is a chain of small dependent Linear layers (4 per layer +
// the LM head) whose weights are fixed; on B200 the chain, not HBM, bounds
// the step when each link is a separate kernel (launch + drain + refill of
// the SMs per link).  Here the chain is kept inside one kernel:
//
//   * warp 0 of every CTA (the producer) walks the whole schedule of weight
//     tiles the CTA will consume -- steps x (layers x {qkv, o, gate|up,
//     down} + LM head), tile t of a matrix to CTA t mod grid -- and streams
//     them with 1-D TMA bulk copies into a ring of shared-memory slots.
//     Weights never depend on activations, so the producer runs ahead
//     across phase, layer and step boundaries, limited only by the ring;
//   * warps 1..16 (the consumers) run the phases in order, separated by a
//     grid-wide barrier: stage the phase's input vector into shared memory
//     (with the fused RMSNorm or SiLU(gate)*up of the engine's decode
//     GEMVs), multiply it with the CTA's resident tiles, write the outputs
//     (bias, residual add or LM-head logits + argmax partial);
//   * attention of head h runs on CTA h, with RoPE of q / k and the KV
//     cache store of the new position folded in;
//   * after the LM head every CTA reduces the per-CTA argmax partials to the
//     next token (lowest index on ties), CTA 0 appends it to the output list
//     and the CTAs write its embedding row as the next step's input.
//
// Per step: 5 grid barriers per layer + 2.  Every wait (ring slots, grid
// barrier) is bounded: on expiry the kernel records B200_DEVICE_TIMEOUT_*
// in the status word, raises a grid-wide abort flag, every CTA leaves its
// loops, waits (bounded) for its bulk copies in flight and returns.
//
// Arithmetic per element is the engine's decode GEMV arithmetic (gemv.cu:
// FP32 accumulation of BF16 x times BF16 w or int8 q * BF16 group scale,
// BF16 rounding of each output, RMSNorm / SiLU / residual roundings of the
// reference, src/cuda/kernels.cu:64-116, 285-324) and the attention of
// attention.cuh.
#include <cfloat>
#include <climits>

#include "attention.cuh"
#include "common.cuh"
#include "gemv_math.cuh"
#include "persistent.h"

namespace b200 {
namespace {

constexpr int kPWarps = 16;                 // consumer warps
constexpr int kPThreads = 32 * (kPWarps + 1);
constexpr int kPConsumers = 32 * kPWarps;   // 512
constexpr int kPSmemLimit = 227 * 1024;
constexpr int kPSlotCap = 32 * 1024;
constexpr int kPMaxStages = 8;
constexpr int kPMaxStageK = 3 * 4 * kPConsumers;  // in_features staged from registers
constexpr int kPMisc = 1024;

__device__ __forceinline__ void cbar() {
  asm volatile("bar.sync 1, %0;" ::"n"(kPConsumers) : "memory");
}

struct Role {
  const void* w;
  const bf16* s;
  int n, k, rpt;
};

__device__ __forceinline__ Role role_of(const PersistArgs& a, const PersistLayer& L,
                                        int role) {
  switch (role) {
    case kRoleQkv:
      return {L.qkv_w, L.qkv_s, (a.heads + 2 * a.kv_heads) * kHeadDim, a.hidden, a.rpt[0]};
    case kRoleO:
      return {L.o_w, L.o_s, a.hidden, a.hidden, a.rpt[1]};
    case kRoleGateUp:
      return {L.gu_w, L.gu_s, 2 * a.inter, a.hidden, a.rpt[2]};
    case kRoleDown:
      return {L.down_w, L.down_s, a.hidden, a.inter, a.rpt[3]};
    default:
      return {a.embed, nullptr, a.vocab, a.hidden, a.rpt[4]};
  }
}

struct Ring {
  int s = 0;        // slot
  uint32_t ph = 0;  // parity of the slot's current use
  int i = 0;        // tiles so far
  int fail = -1;    // consumers: first tile whose wait failed
};

__device__ __forceinline__ void ring_next(Ring& r, int stages) {
  ++r.i;
  if (++r.s == stages) {
    r.s = 0;
    r.ph ^= 1u;
  }
}

struct Smem {
  unsigned char* ring;
  uint32_t bar_full, bar_empty;
  volatile int* abort_flag;  // CTA-local
  int* s_ok;
  int* s_issued;
  int* s_consumed;
  float* red_v;
  int* red_i;
  float* red_part;  // [2][kPWarps]
  float* norm_red;  // [kPWarps]
  float4* xs;       // staging region (also the attention scratch)
};

// ---------------------------------------------------------------- producer
__device__ bool produce_role(const Role& r, bool w8, Ring& ring, const Smem& sm,
                             const PersistArgs& a) {
  const int row_bytes = w8 ? r.k : 2 * r.k;
  const int groups = r.k >> 6;
  const int tiles = r.n / r.rpt;
  const uint32_t wb = uint32_t(r.rpt) * row_bytes;
  const uint32_t sb = w8 ? uint32_t(r.rpt) * groups * 2 : 0u;
  for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
    if (!mbar_wait_bounded(sm.bar_empty + 8 * ring.s, ring.ph ^ 1u, sm.abort_flag,
                           B200_DEVICE_TIMEOUT_PIPELINE, a.status)) {
      return false;
    }
    unsigned char* st = sm.ring + size_t(ring.s) * a.slot_bytes;
    const uint32_t full = sm.bar_full + 8 * ring.s;
    mbar_arrive_expect_tx(full, wb + sb);
    bulk_load(smem_u32(st), static_cast<const unsigned char*>(r.w) + size_t(t) * wb, wb, full);
    if (w8) bulk_load(smem_u32(st + wb), r.s + size_t(t) * r.rpt * groups, sb, full);
    ring_next(ring, a.stages);
  }
  return true;
}

// ------------------------------------------------------------- consumers
// Input staging: xs[p * chunks + c] = x'[c * kEPC + 4p .. +3] (FP32 planes,
// gemv.cu layout), x' = x (mode 0), RMSNorm(x) * w (mode 1) or
// silu(gate) * up from [gate | up] (mode 2).
template <int kEPC>
__device__ __forceinline__ void stage_input(const bf16* in, int k, int mode, const bf16* norm_w,
                                            float eps, const Smem& sm, int ct) {
  const int n4 = k >> 2;
  const int chunks = k / kEPC;
  const int lane = ct & 31, cw = ct >> 5;
  uint2 raw[3];
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const int e4 = ct + j * kPConsumers;
    raw[j] = e4 < n4 ? __ldcg(reinterpret_cast<const uint2*>(in) + e4) : make_uint2(0u, 0u);
  }
  float scale = 1.0f;
  if (mode == 1) {
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      if (ct + j * kPConsumers < n4) {
        const float x0 = bf16_lo(raw[j].x), x1 = bf16_hi(raw[j].x);
        const float x2 = bf16_lo(raw[j].y), x3 = bf16_hi(raw[j].y);
        ss = fmaf(x0, x0, ss);
        ss = fmaf(x1, x1, ss);
        ss = fmaf(x2, x2, ss);
        ss = fmaf(x3, x3, ss);
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (lane == 0) sm.norm_red[cw] = ss;
    cbar();
    float total = 0.0f;
#pragma unroll
    for (int w = 0; w < kPWarps; ++w) total += sm.norm_red[w];
    scale = rsqrtf(total / float(k) + eps);
  }
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const int e4 = ct + j * kPConsumers;
    if (e4 < n4) {
      const int c = (e4 * 4) / kEPC;
      const int p = ((e4 * 4) % kEPC) >> 2;
      float4 v = make_float4(bf16_lo(raw[j].x), bf16_hi(raw[j].x), bf16_lo(raw[j].y),
                             bf16_hi(raw[j].y));
      if (mode == 1) {
        const uint2 wr = reinterpret_cast<const uint2*>(norm_w)[e4];
        v.x = bf16_round(v.x * bf16_lo(wr.x) * scale);
        v.y = bf16_round(v.y * bf16_hi(wr.x) * scale);
        v.z = bf16_round(v.z * bf16_lo(wr.y) * scale);
        v.w = bf16_round(v.w * bf16_hi(wr.y) * scale);
      } else if (mode == 2) {
        const uint2 ur = __ldcg(reinterpret_cast<const uint2*>(in + k) + e4);
        v.x = bf16_round(v.x / (1.0f + expf(-v.x)) * bf16_lo(ur.x));
        v.y = bf16_round(v.y / (1.0f + expf(-v.y)) * bf16_hi(ur.x));
        v.z = bf16_round(v.z / (1.0f + expf(-v.z)) * bf16_lo(ur.y));
        v.w = bf16_round(v.w / (1.0f + expf(-v.w)) * bf16_hi(ur.y));
      }
      sm.xs[p * chunks + c] = v;
    }
  }
  cbar();
}

enum Epilogue { kEpiOut = 0, kEpiResidual = 1, kEpiLm = 2 };

// The CTA's tiles of one matrix: kRPT rows per tile, each row split over
// kPWarps / kRPT warps (partials meet in shared memory).
template <bool kW8, int kRPT>
__device__ __forceinline__ void consume_role(const Role& r, Ring& ring, const Smem& sm,
                                             const PersistArgs& a, int epi, const bf16* bias,
                                             bf16* out, float& best, int& best_index, int ct) {
  constexpr int kEPC = kW8 ? 16 : 8;
  constexpr int kPlanes = kEPC / 4;
  constexpr int kWPR = kPWarps / kRPT;
  constexpr int kSpan = 32 * kWPR;
  const int lane = ct & 31, cw = ct >> 5;
  const int k = r.k;
  const int row_bytes = kW8 ? k : 2 * k;
  const int groups = k >> 6;
  const int chunks = k / kEPC;
  const int tiles = r.n / kRPT;
  const int rl = cw / kWPR, ksub = cw % kWPR;
  const int wb = kRPT * row_bytes;
  for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
    const bool ok = __all_sync(
        0xffffffffu, mbar_wait_bounded(sm.bar_full + 8 * ring.s, ring.ph, sm.abort_flag,
                                       B200_DEVICE_TIMEOUT_PIPELINE, a.status));
    const unsigned char* wt = sm.ring + size_t(ring.s) * a.slot_bytes;
    const unsigned char* wrow = wt + rl * row_bytes;
    const bf16* srow = reinterpret_cast<const bf16*>(wt + wb) + rl * groups;
    float2 acc = f2(0.0f, 0.0f);
    if (ok) {
#pragma unroll 2
      for (int c = ksub * 32 + lane; c < chunks; c += kSpan) {
        float4 xv[kPlanes];
#pragma unroll
        for (int p = 0; p < kPlanes; ++p) xv[p] = sm.xs[p * chunks + c];
        const uint4 wv = *reinterpret_cast<const uint4*>(wrow + c * 16);
        if constexpr (kW8) {
          float2 u = f2(0.0f, 0.0f);
          float2 v = f2(0.0f, 0.0f);
          u = dot4_s8_x2(wv.x, xv[0], u);
          v = dot4_s8_x2(wv.y, xv[1], v);
          u = dot4_s8_x2(wv.z, xv[2], u);
          v = dot4_s8_x2(wv.w, xv[3], v);
          const float sc = __bfloat162float(srow[c >> 2]);
          acc = __ffma2_rn(u, f2(sc, sc), acc);
          acc = __ffma2_rn(v, f2(sc, sc), acc);
        } else {
          acc = dot4_bf16_x2(wv.x, wv.y, xv[0], acc);
          acc = dot4_bf16_x2(wv.z, wv.w, xv[1], acc);
        }
      }
    }
    __syncwarp();
    // A slot whose copy was not seen to land is not handed back: the
    // producer never reuses it, and the exit path waits for it.
    if (ok && lane == 0) mbar_arrive(sm.bar_empty + 8 * ring.s);
    if (!ok && ring.fail < 0) ring.fail = ring.i;
    float v = acc.x + acc.y;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if constexpr (kWPR > 1) {
      float* part = sm.red_part + (ring.i & 1) * kPWarps;
      if (lane == 0) part[cw] = v;
      cbar();
      if (ksub == 0) {
        v = 0.0f;
#pragma unroll
        for (int j = 0; j < kWPR; ++j) v += part[cw + j];
      }
    }
    const int row = t * kRPT + rl;
    if (ok && ksub == 0 && lane == 0) {
      if (epi == kEpiResidual) {
        const bf16 y = __float2bfloat16_rn(v);
        const float xr = __bfloat162float(__ushort_as_bfloat16(
            __ldcg(reinterpret_cast<const unsigned short*>(out) + row)));
        out[row] = __float2bfloat16_rn(xr + __bfloat162float(y));
      } else {
        const float b = bias ? __bfloat162float(bias[row]) : 0.0f;
        const bf16 y = __float2bfloat16_rn(v + b);
        out[row] = y;
        if (epi == kEpiLm) argmax_update(best, best_index, __bfloat162float(y), row);
      }
    }
    ring_next(ring, a.stages);
  }
}

template <bool kW8>
__device__ __forceinline__ void consume_any(const Role& r, Ring& ring, const Smem& sm,
                                            const PersistArgs& a, int epi, const bf16* bias,
                                            bf16* out, float& best, int& best_index, int ct) {
  switch (r.rpt) {
    case 16:
      consume_role<kW8, 16>(r, ring, sm, a, epi, bias, out, best, best_index, ct);
      break;
    case 8:
      consume_role<kW8, 8>(r, ring, sm, a, epi, bias, out, best, best_index, ct);
      break;
    case 4:
      consume_role<kW8, 4>(r, ring, sm, a, epi, bias, out, best, best_index, ct);
      break;
    default:
      consume_role<kW8, 2>(r, ring, sm, a, epi, bias, out, best, best_index, ct);
      break;
  }
}

// Grid-wide barrier among the consumers of all CTAs (monotonic counter;
// `target` lives in consumer thread 0).  False: the kernel is aborting.
__device__ __forceinline__ bool grid_sync(const PersistArgs& a, const Smem& sm,
                                          unsigned& target, int ct) {
  cbar();
  if (ct == 0) {
    bool ok = *sm.abort_flag == 0;
    target += gridDim.x;
    const unsigned idx = target / gridDim.x - 1;
    const bool trace = a.trace != nullptr && idx < unsigned(a.trace_count);
    if (trace) a.trace[(size_t(blockIdx.x) * a.trace_count + idx) * 2] = global_timer_ns();
    if (ok) {
      __threadfence();
      atomicAdd(a.grid_counter, 1u);
      const uint64_t start = global_timer_ns();
      while (true) {
        unsigned v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a.grid_counter)
                     : "memory");
        if (int(v - target) >= 0) break;
        if (*reinterpret_cast<volatile int*>(a.grid_abort) != 0) {
          ok = false;
          break;
        }
        if (global_timer_ns() - start > kWaitTimeoutNs) {
          atomicCAS(a.status, 0, B200_DEVICE_TIMEOUT_GRID);
          ok = false;
          break;
        }
      }
      __threadfence();
    }
    if (trace) a.trace[(size_t(blockIdx.x) * a.trace_count + idx) * 2 + 1] = global_timer_ns();
    if (!ok) {
      atomicExch(a.grid_abort, 1);
      *sm.abort_flag = 1;
    }
    *sm.s_ok = ok ? 1 : 0;
  }
  cbar();
  return *sm.s_ok != 0;
}

// Embedding row of `tok` as the residual stream (each CTA a slice).
__device__ __forceinline__ void write_embedding(const PersistArgs& a, int tok, int ct) {
  const uint4* src = reinterpret_cast<const uint4*>(a.embed + size_t(tok) * a.hidden);
  uint4* dst = reinterpret_cast<uint4*>(a.x);
  for (int j = blockIdx.x * kPConsumers + ct; j < a.hidden / 8; j += gridDim.x * kPConsumers) {
    dst[j] = src[j];
  }
}

// Attention of head blockIdx.x for the token at `pos` of layer `l`, with
// RoPE (half-split pairs, frequency theta^(-2i/64)) of q and k and the
// cache store of k / v at `pos` by the first head of each KV group.
__device__ __forceinline__ void attention_phase(const PersistArgs& a, const Smem& sm, int l,
                                                int pos, int ct) {
  const int h = blockIdx.x;
  const int group = a.heads / a.kv_heads;
  const int kvh = h / group;
  float* qs = reinterpret_cast<float*>(sm.xs);
  float* kcur = qs + kHeadDim;
  float* vcur = kcur + kHeadDim;
  float* scratch = vcur + kHeadDim;
  const size_t cache_off = (size_t(l) * a.kv_heads + kvh) * a.max_seq * kHeadDim;
  bf16* kc = a.kcache + cache_off;
  bf16* vc = a.vcache + cache_off;
  const bool writer = h % group == 0;
  const unsigned short* row = reinterpret_cast<const unsigned short*>(a.qkv);
  constexpr int half = kHeadDim / 2;
  auto ld = [&](int idx) { return __bfloat162float(__ushort_as_bfloat16(__ldcg(row + idx))); };
  if (ct < 2 * half) {
    const int i = ct % half;
    const bool is_k = ct >= half;
    const int base = is_k ? (a.heads + kvh) * kHeadDim : h * kHeadDim;
    const float freq = powf(a.theta, -2.0f * float(i) / float(kHeadDim));
    float sn, cs;
    sincosf(float(pos) * freq, &sn, &cs);
    const float x0 = ld(base + i), x1 = ld(base + i + half);
    const bf16 r0 = __float2bfloat16_rn(x0 * cs - x1 * sn);
    const bf16 r1 = __float2bfloat16_rn(x1 * cs + x0 * sn);
    float* dst = is_k ? kcur : qs;
    dst[i] = __bfloat162float(r0);
    dst[i + half] = __bfloat162float(r1);
    if (is_k && writer) {
      kc[size_t(pos) * kHeadDim + i] = r0;
      kc[size_t(pos) * kHeadDim + i + half] = r1;
    }
  } else if (ct < 2 * half + kHeadDim) {
    const int d = ct - 2 * half;
    const int idx = (a.heads + a.kv_heads + kvh) * kHeadDim + d;
    const unsigned short bits = __ldcg(row + idx);
    vcur[d] = __bfloat162float(__ushort_as_bfloat16(bits));
    if (writer) vc[size_t(pos) * kHeadDim + d] = __ushort_as_bfloat16(bits);
  }
  cbar();
  attend_row<kPConsumers>(qs, kc, vc, pos + 1, pos, kcur, vcur, scratch, ct, [] { cbar(); },
                          a.att + h * kHeadDim);
}

template <bool kW8>
__global__ void __launch_bounds__(kPThreads, 1) decode_persistent_kernel(const PersistArgs a) {
  extern __shared__ __align__(128) unsigned char psmem[];
  Smem sm;
  sm.ring = psmem;
  sm.xs = reinterpret_cast<float4*>(psmem + a.region_off);
  uint64_t* bars = reinterpret_cast<uint64_t*>(psmem + a.bars_off);
  sm.bar_full = smem_u32(bars);
  sm.bar_empty = sm.bar_full + 8 * a.stages;
  int* misc = reinterpret_cast<int*>(bars + 2 * a.stages);
  sm.abort_flag = misc;
  sm.s_ok = misc + 1;
  sm.s_issued = misc + 2;
  sm.s_consumed = misc + 3;
  sm.red_v = reinterpret_cast<float*>(misc + 4);
  sm.red_i = misc + 4 + kPWarps;
  sm.red_part = reinterpret_cast<float*>(misc + 4 + 2 * kPWarps);
  sm.norm_red = sm.red_part + 2 * kPWarps;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(sm.bar_full + 8 * s, 1);
      mbar_init(sm.bar_empty + 8 * s, kPWarps);
    }
    *sm.abort_flag = 0;
    *sm.s_issued = 0;
    *sm.s_consumed = INT_MAX;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == 0) {
    if (lane == 0) {
      Ring ring;
      bool ok = true;
      for (int step = 0; step < a.steps && ok; ++step) {
        for (int l = 0; l < a.n_layers && ok; ++l) {
          const PersistLayer L = a.layers[l];
          for (int role = kRoleQkv; role <= kRoleDown && ok; ++role) {
            ok = produce_role(role_of(a, L, role), kW8, ring, sm, a);
          }
        }
        if (ok) ok = produce_role(role_of(a, a.layers[0], kRoleLm), false, ring, sm, a);
      }
      *sm.s_issued = ring.i;
    }
  } else {
    const int ct = threadIdx.x - 32;
    const int pos0 = *a.d_pos;
    const int step0 = *a.d_step;
    int tok = *a.d_token;
    unsigned target = 0;
    Ring ring;
    float best = -FLT_MAX;
    int best_index = INT_MAX;
    const int H = a.hidden;
    write_embedding(a, tok, ct);
    bool alive = grid_sync(a, sm, target, ct);
    int step = 0;
    for (; step < a.steps && alive; ++step) {
      const int pos = pos0 + step;
      for (int l = 0; l < a.n_layers && alive; ++l) {
        const PersistLayer L = a.layers[l];
        // q | k | v = W_qkv RMSNorm(x) + b
        stage_input<kW8 ? 16 : 8>(a.x, H, 1, L.in_norm, a.eps, sm, ct);
        consume_any<kW8>(role_of(a, L, kRoleQkv), ring, sm, a, kEpiOut, L.qkv_b, a.qkv, best,
                         best_index, ct);
        if (!(alive = grid_sync(a, sm, target, ct))) break;
        if (int(blockIdx.x) < a.heads) attention_phase(a, sm, l, pos, ct);
        if (!(alive = grid_sync(a, sm, target, ct))) break;
        // x += W_o att
        stage_input<kW8 ? 16 : 8>(a.att, H, 0, nullptr, 0.0f, sm, ct);
        consume_any<kW8>(role_of(a, L, kRoleO), ring, sm, a, kEpiResidual, nullptr, a.x, best,
                         best_index, ct);
        if (!(alive = grid_sync(a, sm, target, ct))) break;
        // gate | up = W_gu RMSNorm(x)
        stage_input<kW8 ? 16 : 8>(a.x, H, 1, L.post_norm, a.eps, sm, ct);
        consume_any<kW8>(role_of(a, L, kRoleGateUp), ring, sm, a, kEpiOut, nullptr, a.gu, best,
                         best_index, ct);
        if (!(alive = grid_sync(a, sm, target, ct))) break;
        // x += W_down (silu(gate) * up)
        stage_input<kW8 ? 16 : 8>(a.gu, a.inter, 2, nullptr, 0.0f, sm, ct);
        consume_any<kW8>(role_of(a, L, kRoleDown), ring, sm, a, kEpiResidual, nullptr, a.x,
                         best, best_index, ct);
        alive = grid_sync(a, sm, target, ct);
      }
      if (!alive) break;
      // logits = E RMSNorm(x), per-CTA argmax partial
      stage_input<8>(a.x, H, 1, a.final_norm, a.eps, sm, ct);
      best = -FLT_MAX;
      best_index = INT_MAX;
      consume_any<false>(role_of(a, a.layers[0], kRoleLm), ring, sm, a, kEpiLm, nullptr,
                         a.logits, best, best_index, ct);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, off);
        const int oi = __shfl_xor_sync(0xffffffffu, best_index, off);
        argmax_update(best, best_index, ov, oi);
      }
      if (lane == 0) {
        sm.red_v[ct >> 5] = best;
        sm.red_i[ct >> 5] = best_index;
      }
      cbar();
      if (ct == 0) {
        float b = -FLT_MAX;
        int bi = INT_MAX;
        for (int w = 0; w < kPWarps; ++w) argmax_update(b, bi, sm.red_v[w], sm.red_i[w]);
        a.part_v[blockIdx.x] = b;
        a.part_i[blockIdx.x] = bi;
      }
      if (!(alive = grid_sync(a, sm, target, ct))) break;
      // next token: argmax over the CTAs' partials
      float b = -FLT_MAX;
      int bi = INT_MAX;
      for (int j = ct; j < int(gridDim.x); j += kPConsumers) {
        argmax_update(b, bi, __ldcg(a.part_v + j), __ldcg(a.part_i + j));
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, b, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        argmax_update(b, bi, ov, oi);
      }
      if (lane == 0) {
        sm.red_v[ct >> 5] = b;
        sm.red_i[ct >> 5] = bi;
      }
      cbar();
      b = -FLT_MAX;
      bi = INT_MAX;
      for (int w = 0; w < kPWarps; ++w) argmax_update(b, bi, sm.red_v[w], sm.red_i[w]);
      tok = bi == INT_MAX ? 0 : bi;
      if (blockIdx.x == 0 && ct == 0 && step0 + step < a.max_out) a.d_out[step0 + step] = tok;
      write_embedding(a, tok, ct);
      alive = grid_sync(a, sm, target, ct);
    }
    if (lane == 0) atomicMin(sm.s_consumed, ring.fail >= 0 ? ring.fail : ring.i);
    if (ct == 0) {
      if (!alive) *sm.abort_flag = 1;  // ends the producer's waits
      if (alive && blockIdx.x == 0) {
        *a.d_pos = pos0 + a.steps;
        *a.d_step = step0 + a.steps;
        *a.d_token = tok;
      }
    }
  }
  __syncthreads();
  // After an abort: wait (bounded) for the bulk copies still in flight into
  // this CTA's ring before the CTA exits (at most one per slot: a slot is
  // reissued only after all consumer warps saw its previous copy land).
  if (threadIdx.x == 0) {
    for (int j = *sm.s_consumed; j < *sm.s_issued; ++j) {
      const int s = j % a.stages;
      const uint32_t parity = uint32_t(j / a.stages) & 1u;
      const uint64_t start = global_timer_ns();
      while (!mbar_try_wait(sm.bar_full + 8 * s, parity)) {
        if (global_timer_ns() - start > kWaitTimeoutNs) break;
      }
    }
  }
}

int sm_count() {
  int dev = 0, count = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev);
  return count;
}

// Rows per tile of an n x k matrix: the smallest estimated time of the
// busiest CTA (tiles per CTA x (row work + a fixed per-tile cost)) among
// tiles that fit a ring slot and keep the 1-D copies 16-byte aligned.
int pick_rpt(int n, int k, bool w8, int grid) {
  int best = 0;
  double best_cost = 1e30;
  for (int rpt : {16, 8, 4, 2}) {
    if (n % rpt != 0) continue;
    const int row_bytes = w8 ? k : 2 * k;
    const int sb = w8 ? rpt * (k / 64) * 2 : 0;
    if (sb % 16 != 0) continue;
    if (rpt * row_bytes + sb > kPSlotCap) continue;
    const int tiles = n / rpt;
    const int per = (tiles + grid - 1) / grid;
    const double cost = per * (rpt * (k / 1024.0) + 3.0);
    if (cost < best_cost * 0.999) {
      best_cost = cost;
      best = rpt;
    }
  }
  return best;
}

}  // namespace

PersistPlan plan_persistent(bool w8, int hidden, int inter, int heads, int kv_heads, int vocab,
                            int max_seq) {
  PersistPlan p;
  if (hidden % 64 != 0 || inter % 64 != 0 || hidden > kPMaxStageK || inter > kPMaxStageK ||
      heads * kHeadDim != hidden || heads % kv_heads != 0 || max_seq <= 0) {
    return p;
  }
  const int grid = sm_count();
  if (heads > grid) return p;
  const int n[5] = {(heads + 2 * kv_heads) * kHeadDim, hidden, 2 * inter, hidden, vocab};
  const int k[5] = {hidden, hidden, hidden, inter, hidden};
  int slot = 0;
  for (int r = 0; r < 5; ++r) {
    const bool rw8 = w8 && r != kRoleLm;
    p.rpt[r] = pick_rpt(n[r], k[r], rw8, grid);
    if (p.rpt[r] == 0) return p;
    const int row_bytes = rw8 ? k[r] : 2 * k[r];
    const int bytes = p.rpt[r] * row_bytes + (rw8 ? p.rpt[r] * (k[r] / 64) * 2 : 0);
    slot = bytes > slot ? bytes : slot;
  }
  slot = (slot + 127) / 128 * 128;
  const size_t stage_bytes = size_t(hidden > inter ? hidden : inter) * 4;
  const size_t att_bytes = (attend_smem_floats<kPConsumers>(max_seq) + 3 * kHeadDim) * 4;
  const int region = int(((stage_bytes > att_bytes ? stage_bytes : att_bytes) + 127) / 128 * 128);
  const int avail = kPSmemLimit - region - kPMisc - 16 * kPMaxStages;
  int stages = avail / slot;
  if (stages > kPMaxStages) stages = kPMaxStages;
  if (stages < 2) return p;
  p.slot_bytes = slot;
  p.stages = stages;
  p.region_off = stages * slot;
  p.bars_off = p.region_off + region;
  p.smem = p.bars_off + 16 * stages + kPMisc;
  auto kernel = w8 ? decode_persistent_kernel<true> : decode_persistent_kernel<false>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, p.smem) !=
      cudaSuccess) {
    cudaGetLastError();
    return p;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kPThreads, p.smem) !=
          cudaSuccess ||
      per_sm < 1) {
    cudaGetLastError();
    return p;
  }
  p.grid = grid;
  p.ok = true;
  return p;
}

cudaError_t launch_persistent(bool w8, const PersistPlan& plan, const PersistArgs& args,
                              cudaStream_t stream) {
  if (!plan.ok) return cudaErrorInvalidConfiguration;
  PersistArgs a = args;
  a.stages = plan.stages;
  a.slot_bytes = plan.slot_bytes;
  a.region_off = plan.region_off;
  a.bars_off = plan.bars_off;
  for (int r = 0; r < 5; ++r) a.rpt[r] = plan.rpt[r];
  // grid_counter and grid_abort are adjacent words.
  cudaError_t e = cudaMemsetAsync(a.grid_counter, 0, 8, stream);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan.grid);
  cfg.blockDim = dim3(kPThreads);
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return w8 ? cudaLaunchKernelEx(&cfg, decode_persistent_kernel<true>, a)
            : cudaLaunchKernelEx(&cfg, decode_persistent_kernel<false>, a);
}

}  // namespace b200
