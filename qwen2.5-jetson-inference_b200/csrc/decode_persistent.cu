// Persistent decode kernel: every greedy decode step of the Qwen2.5 model
// (all layers, the LM head and the argmax) in one cooperative launch, one
// CTA per SM, for any number of steps.
//
// A decode step is a chain of small dependent matrix-vector products (4 per
// layer + the LM head) over fixed weights.  Launched as separate kernels,
// each link of the chain pays a launch, a drain of the SMs and a refill of
// its weight stream; here the chain stays inside one kernel:
//
//   * Weights.  Each CTA owns a fixed share of every matrix: a contiguous
//     block of rows of q|k|v, o_proj and down_proj, the matching gate and
//     up rows of gate|up (so that silu(gate) * up is formed in the
//     epilogue), and LM-head tiles round-robin.  Warp 0 (the producer) walks
//     that schedule over all steps and streams each block with 1-D TMA bulk
//     copies into a byte ring in shared memory (8 block descriptors with
//     full / empty mbarriers).  Weights never depend on activations, so the
//     producer runs ahead across layer and step boundaries, bounded only by
//     the ring.
//   * Activations flow through tagged 64-bit words in global memory (BF16
//     value bits | 32-bit step tag), one buffer per layer and tensor, each
//     written once per step.  A consumer stage reads its input vector until
//     every word carries the current step's tag: the data is its own
//     barrier, so no grid-wide barrier is needed and a CTA starts a phase as
//     soon as its inputs exist.
//   * Warps 1..16 (the consumers) run, per layer: RMSNorm(x) -> q|k|v (+b);
//     attention of head h on CTA h (RoPE of q and k, KV-cache store of the
//     new position, attention over the cache); o_proj + residual;
//     RMSNorm -> gate|up -> silu(gate) * up; down_proj + residual.  Then the
//     final RMSNorm and the LM head (BF16 logits + per-CTA argmax partial),
//     and every CTA reduces the partials to the next token (lowest index on
//     ties), whose embedding row is the next step's input.
//
// Every wait (ring, tagged words) is bounded: on expiry the kernel records
// B200_DEVICE_TIMEOUT_* in the status word, raises a grid-wide abort flag
// that every other wait checks, leaves its loops, waits (bounded) for its
// bulk copies in flight and returns.
//
// Arithmetic per element is the engine's decode arithmetic (gemv.cu: FP32
// accumulation of BF16 x times BF16 w or int8 q * BF16 group scale, BF16
// rounding of each output; RMSNorm / SiLU / residual roundings of the
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

using u64 = unsigned long long;

constexpr int kPWarps = 16;                 // consumer warps
constexpr int kPThreads = 32 * (kPWarps + 1);
constexpr int kPConsumers = 32 * kPWarps;   // 512
constexpr int kPSmemLimit = 227 * 1024;
constexpr int kNDesc = 8;                   // blocks in flight per CTA
constexpr int kPMaxStageK = 3 * 4 * kPConsumers;  // in_features staged from registers
constexpr int kPMaxBias = 128;
constexpr int kPMisc = 2048;

__device__ __forceinline__ void cbar() {
  asm volatile("bar.sync 1, %0;" ::"n"(kPConsumers) : "memory");
}
// Consumer barrier that also ORs a predicate over the consumer threads.
__device__ __forceinline__ bool cbar_or(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(uint32_t(v)), "n"(kPConsumers)
      : "memory");
  return r != 0;
}

// ------------------------------------------------------------ tagged words
__device__ __forceinline__ u64 tag_word(bf16 v, unsigned tag) {
  return (u64(tag) << 32) | u64(__bfloat16_as_ushort(v));
}
__device__ __forceinline__ void st_word(u64* p, u64 w) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ u64 ld_word(const u64* p) {
  u64 w;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}
__device__ __forceinline__ void ld_word2(const u64* p, u64& a, u64& b) {
  asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];"
               : "=l"(a), "=l"(b)
               : "l"(p)
               : "memory");
}
__device__ __forceinline__ unsigned tag_of(u64 w) { return unsigned(w >> 32); }
__device__ __forceinline__ uint32_t lo16(u64 w) { return uint32_t(w) & 0xffffu; }

struct Smem {
  unsigned char* ring;
  uint32_t bar_full, bar_empty;  // [kNDesc] each
  int* desc_off;                 // [kNDesc] ring offsets of the blocks
  volatile int* abort_flag;      // CTA-local
  int* s_issued;
  int* s_consumed;
  float* red_v;                  // [kPWarps]
  int* red_i;                    // [kPWarps]
  float* red_part;               // [2][2][kPWarps]
  float* norm_red;               // [kPWarps]
  float* bias_s;                 // [kPMaxBias] this CTA's q|k|v bias
  float4* xs;                    // staging region (also the attention scratch)
  bf16* x_layer;                 // [hidden] x entering the layer
  bf16* x_mid;                   // [hidden] x after o_proj
};

// Bounded spin bookkeeping: every 32 spins checks the abort flags and the
// clock; false = give up (the flags are raised).
struct Spin {
  uint64_t start = 0;
  int n = 0;
};
__device__ __forceinline__ bool spin_on(Spin& s, const PersistArgs& a, const Smem& sm) {
  // No sleep between polls: with __nanosleep(64) here decode ran at 2157
  // tok/s, without it 2241 (input staging 1.0 -> 0.67 us per phase).
  if ((++s.n & 31) != 0) return true;
  if (*reinterpret_cast<volatile int*>(a.grid_abort) != 0 || *sm.abort_flag != 0) {
    *sm.abort_flag = 1;
    return false;
  }
  const uint64_t now = global_timer_ns();
  if (s.start == 0) {
    s.start = now;
  } else if (now - s.start > kWaitTimeoutNs) {
    atomicCAS(a.status, 0, B200_DEVICE_TIMEOUT_GRID);
    atomicExch(a.grid_abort, 1);
    *sm.abort_flag = 1;
    return false;
  }
  return true;
}

__device__ __forceinline__ bool wait_word(const u64* p, unsigned tag, u64& w,
                                          const PersistArgs& a, const Smem& sm) {
  Spin s;
  while (true) {
    w = ld_word(p);
    if (tag_of(w) == tag) return true;
    if (!spin_on(s, a, sm)) return false;
  }
}

// Two tagged words, both loads issued before either tag is checked.
__device__ __forceinline__ bool wait_word2(const u64* p0, const u64* p1, unsigned tag, u64& w0,
                                           u64& w1, const PersistArgs& a, const Smem& sm) {
  Spin s;
  w0 = ld_word(p0);
  w1 = ld_word(p1);
  while (true) {
    const bool h0 = tag_of(w0) == tag, h1 = tag_of(w1) == tag;
    if (h0 && h1) return true;
    if (!spin_on(s, a, sm)) return false;
    if (!h0) w0 = ld_word(p0);
    if (!h1) w1 = ld_word(p1);
  }
}

// Up to three groups of four tagged words (groups ct, ct + 512, ct + 1024 of
// `words`, n4 groups in all): all loads are issued before any tag is
// checked, and only groups not yet tagged are read again.
__device__ __forceinline__ bool wait_groups(const u64* words, int ct, int n4, unsigned tag,
                                            uint2 (&out)[3], const PersistArgs& a,
                                            const Smem& sm) {
  u64 w[3][4];
  bool have[3];
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const int e4 = ct + j * kPConsumers;
    have[j] = e4 >= n4;
    if (!have[j]) {
      ld_word2(words + 4 * e4, w[j][0], w[j][1]);
      ld_word2(words + 4 * e4 + 2, w[j][2], w[j][3]);
    } else {
      w[j][0] = w[j][1] = w[j][2] = w[j][3] = 0;
    }
  }
  Spin s;
  bool ok = true;
  while (true) {
    bool all = true;
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      if (!have[j]) {
        have[j] = tag_of(w[j][0]) == tag && tag_of(w[j][1]) == tag &&
                  tag_of(w[j][2]) == tag && tag_of(w[j][3]) == tag;
        all = all && have[j];
      }
    }
    if (all) break;
    if (!spin_on(s, a, sm)) {
      ok = false;
      break;
    }
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      if (!have[j]) {
        const u64* p = words + 4 * (ct + j * kPConsumers);
        ld_word2(p, w[j][0], w[j][1]);
        ld_word2(p + 2, w[j][2], w[j][3]);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    out[j].x = lo16(w[j][0]) | (lo16(w[j][1]) << 16);
    out[j].y = lo16(w[j][2]) | (lo16(w[j][3]) << 16);
  }
  return ok;
}

// -------------------------------------------------------------- schedule
struct Block {
  const unsigned char* w[2];
  const bf16* s[2];
  int parts;  // 2: [gate rows; up rows]
  int rows;   // rows per part (outputs of the block)
  int row0;   // first output row
  int k;
  bool w8;
};

__device__ __forceinline__ uint32_t block_bytes(const Block& b) {
  const uint32_t row = b.w8 ? uint32_t(b.k) : 2u * b.k;
  const uint32_t srow = b.w8 ? uint32_t(b.k >> 6) * 2u : 0u;
  return uint32_t(b.parts) * b.rows * (row + srow);
}

// Sub-block `t` of the CTA's share of a layer matrix (rows == 0: none), or
// LM-head tile t.
__device__ __forceinline__ Block block_of(const PersistArgs& a, const PersistLayer& L, int role,
                                          bool w8, int t) {
  Block b;
  b.parts = 1;
  b.w8 = w8;
  int n = 0, per = 0;
  const void* w = nullptr;
  const bf16* s = nullptr;
  switch (role) {
    case kRoleQkv:
      n = (a.heads + 2 * a.kv_heads) * kHeadDim;
      b.k = a.hidden;
      w = L.qkv_w;
      s = L.qkv_s;
      per = a.rows[kRoleQkv];
      break;
    case kRoleO:
      n = a.hidden;
      b.k = a.hidden;
      w = L.o_w;
      s = L.o_s;
      per = a.rows[kRoleO];
      break;
    case kRoleGateUp:
      n = a.inter;
      b.k = a.hidden;
      w = L.gu_w;
      s = L.gu_s;
      per = a.rows[kRoleGateUp];
      b.parts = 2;
      break;
    case kRoleDown:
      n = a.hidden;
      b.k = a.inter;
      w = L.down_w;
      s = L.down_s;
      per = a.rows[kRoleDown];
      break;
    default:
      n = a.vocab;
      b.k = a.hidden;
      w = a.embed;
      per = a.lm_rows;
      b.w8 = false;
      break;
  }
  if (role == kRoleLm) {
    b.row0 = t * per;
    b.rows = b.row0 < n ? min(per, n - b.row0) : 0;
  } else {
    const int sub = a.sub_rows[role];
    const int share0 = int(blockIdx.x) * per;
    const int share1 = min(n, share0 + per);
    b.row0 = share0 + t * sub;
    b.rows = b.row0 < share1 ? min(sub, share1 - b.row0) : 0;
  }
  const size_t row_bytes = b.w8 ? size_t(b.k) : 2 * size_t(b.k);
  const int groups = b.k >> 6;
  for (int p = 0; p < 2; ++p) {
    const size_t r = size_t(b.row0) + size_t(p) * n;  // up rows follow the gate rows
    b.w[p] = static_cast<const unsigned char*>(w) + r * row_bytes;
    b.s[p] = b.w8 ? s + r * groups : nullptr;
  }
  return b;
}

// ---------------------------------------------------------------- producer
struct Producer {
  int j = 0;        // blocks issued
  int o = 0;        // oldest block not known consumed
  long long P = 0;  // ring bytes issued (monotonic, with wrap padding)
  long long C = 0;  // ring bytes released
  long long end[kNDesc];
};

__device__ bool produce(const Block& b, Producer& pr, const Smem& sm, const PersistArgs& a) {
  if (b.rows == 0) return true;
  const uint32_t bytes = block_bytes(b);
  const long long R = a.ring_bytes;
  long long pos = pr.P;
  if (pos % R + bytes > R) pos += R - pos % R;  // blocks are contiguous in the ring
  while (pr.j - pr.o >= kNDesc || pos + bytes - pr.C > R) {
    const int d = pr.o % kNDesc;
    if (!mbar_wait_bounded(sm.bar_empty + 8 * d, uint32_t(pr.o / kNDesc) & 1u, sm.abort_flag,
                           B200_DEVICE_TIMEOUT_PIPELINE, a.status)) {
      return false;
    }
    pr.C = pr.end[d];
    ++pr.o;
  }
  const int d = pr.j % kNDesc;
  const int off = int(pos % R);
  sm.desc_off[d] = off;
  pr.end[d] = pos + bytes;
  const uint32_t full = sm.bar_full + 8 * d;
  mbar_arrive_expect_tx(full, bytes);
  const uint32_t row = b.w8 ? uint32_t(b.k) : 2u * b.k;
  const uint32_t wpart = uint32_t(b.rows) * row;
  const uint32_t spart = b.w8 ? uint32_t(b.rows) * uint32_t(b.k >> 6) * 2u : 0u;
  unsigned char* dst = sm.ring + off;
  for (int p = 0; p < b.parts; ++p) bulk_load(smem_u32(dst + p * wpart), b.w[p], wpart, full);
  if (b.w8) {
    dst += b.parts * wpart;
    for (int p = 0; p < b.parts; ++p) bulk_load(smem_u32(dst + p * spart), b.s[p], spart, full);
  }
  pr.P = pos + bytes;
  ++pr.j;
  return true;
}

// ------------------------------------------------------------- consumers
struct Consumer {
  int j = 0;       // blocks taken
  int fail = -1;   // first block whose wait failed
  int red_it = 0;  // reduction buffer parity counter
};

__device__ __forceinline__ bool acquire(Consumer& cs, const Smem& sm, const PersistArgs& a,
                                        const unsigned char*& blk) {
  const int d = cs.j % kNDesc;
  const bool ok = __all_sync(
      0xffffffffu, mbar_wait_bounded(sm.bar_full + 8 * d, uint32_t(cs.j / kNDesc) & 1u,
                                     sm.abort_flag, B200_DEVICE_TIMEOUT_PIPELINE, a.status));
  blk = sm.ring + sm.desc_off[d];
  if (!ok && cs.fail < 0) cs.fail = cs.j;
  return ok;
}

// A block whose copy was not seen to land is not handed back: the producer
// never reuses its bytes and the exit path waits for it.
__device__ __forceinline__ void release(Consumer& cs, const Smem& sm, bool ok, int lane) {
  __syncwarp();
  if (ok && lane == 0) mbar_arrive(sm.bar_empty + 8 * (cs.j % kNDesc));
  ++cs.j;
}

// Input staging: xs[p * chunks + c] = x'[c * kEPC + 4p .. +3] (FP32 planes,
// gemv.cu layout) with x' = x or bf16(x * w * rsqrt(mean(x^2) + eps)).  x is
// read from tagged words (waiting for `tag`) or from plain BF16; raw_out
// (optional, shared memory) receives x itself.  Returns false (uniformly)
// when the kernel is aborting.
template <int kEPC>
__device__ __forceinline__ bool stage(const u64* words, const bf16* plain, unsigned tag, int k,
                                      const bf16* norm_w, float eps, bf16* raw_out,
                                      const PersistArgs& a, const Smem& sm, int ct, int phase) {
  const int n4 = k >> 2;
  const int chunks = k / kEPC;
  const int lane = ct & 31, cw = ct >> 5;
  // Norm gains first: they do not depend on the input, so their load
  // overlaps the wait for it.
  uint2 gain[3];
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const int e4 = ct + j * kPConsumers;
    gain[j] = norm_w != nullptr && e4 < n4 ? reinterpret_cast<const uint2*>(norm_w)[e4]
                                           : make_uint2(0u, 0u);
  }
  uint2 raw[3];
  if (words != nullptr) {
    wait_groups(words, ct, n4, tag, raw, a, sm);
    if (a.trace != nullptr && ct == 0 && phase < a.trace_count) {
      a.trace[(size_t(blockIdx.x) * a.trace_count + phase) * 4 + 3] = global_timer_ns();
    }
  } else {
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const int e4 = ct + j * kPConsumers;
      raw[j] = e4 < n4 ? reinterpret_cast<const uint2*>(plain)[e4] : make_uint2(0u, 0u);
    }
  }
  if (raw_out != nullptr) {
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const int e4 = ct + j * kPConsumers;
      if (e4 < n4) reinterpret_cast<uint2*>(raw_out)[e4] = raw[j];
    }
  }
  float scale = 1.0f;
  if (norm_w != nullptr) {
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const float x0 = bf16_lo(raw[j].x), x1 = bf16_hi(raw[j].x);
      const float x2 = bf16_lo(raw[j].y), x3 = bf16_hi(raw[j].y);
      ss = fmaf(x0, x0, ss);
      ss = fmaf(x1, x1, ss);
      ss = fmaf(x2, x2, ss);
      ss = fmaf(x3, x3, ss);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (lane == 0) sm.norm_red[cw] = ss;
    cbar();  // also: every warp is done reading the previous staged vector
    float total = 0.0f;
#pragma unroll
    for (int w = 0; w < kPWarps; ++w) total += sm.norm_red[w];
    scale = rsqrtf(total / float(k) + eps);
  } else {
    cbar();  // every warp is done reading the previous phase's staged vector
  }
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const int e4 = ct + j * kPConsumers;
    if (e4 < n4) {
      const int c = (e4 * 4) / kEPC;
      const int p = ((e4 * 4) % kEPC) >> 2;
      float4 v = make_float4(bf16_lo(raw[j].x), bf16_hi(raw[j].x), bf16_lo(raw[j].y),
                             bf16_hi(raw[j].y));
      if (norm_w != nullptr) {
        const uint2 wr = gain[j];
        v.x = bf16_round(v.x * bf16_lo(wr.x) * scale);
        v.y = bf16_round(v.y * bf16_hi(wr.x) * scale);
        v.z = bf16_round(v.z * bf16_lo(wr.y) * scale);
        v.w = bf16_round(v.w * bf16_hi(wr.y) * scale);
      }
      sm.xs[p * chunks + c] = v;
    }
  }
  return !cbar_or(*sm.abort_flag != 0);
}

// Products of one block with the staged vector.  Output o of the block is
// row o (kPair: rows o and rows + o, the gate and up rows).  Each output is
// computed by kLPR lanes of one warp (kWPR == 1, several outputs per warp)
// or by kWPR whole warps (kLPR == 32, partials meet in shared memory); a
// lane takes the 16-byte chunks c = first, first + kLPR * kWPR, ...
// kK != 0 compiles the loop for that in_features (fully unrolled, every
// chunk load issued up front); kK == 0 takes any in_features.
// epi(o, vA, vB) runs on one lane per output.
template <bool kW8, int kK, int kLPR, int kWPR, bool kPair, class Epi>
__device__ __forceinline__ void gemv_block(const unsigned char* blk, bool ok, int rows, int k,
                                           Consumer& cs, const Smem& sm, int ct, Epi epi) {
  static_assert(kWPR == 1 || kLPR == 32, "split outputs use whole warps");
  constexpr int kEPC = kW8 ? 16 : 8;
  constexpr int kPlanes = kEPC / 4;
  constexpr int kRG = kWPR > 1 ? 1 : 32 / kLPR;               // outputs per warp
  constexpr int kOutIt = kWPR > 1 ? kPWarps / kWPR : kPWarps * kRG;
  constexpr int kSpan = kLPR * kWPR;                          // lanes per output
  constexpr int kChunksK = kK / kEPC;
  constexpr int kIt = kK != 0 ? (kChunksK + kSpan - 1) / kSpan : 0;
  const int lane = ct & 31, cw = ct >> 5;
  const int ll = lane % kLPR;
  const int ksub = kWPR > 1 ? cw % kWPR : 0;
  const int slot = kWPR > 1 ? cw / kWPR : cw * kRG + lane / kLPR;
  const int first = ksub * 32 + ll;
  const int row_bytes = kW8 ? k : 2 * k;
  const int groups = k >> 6;
  const int chunks = kK != 0 ? kChunksK : k / kEPC;
  const int total_rows = kPair ? 2 * rows : rows;
  const bf16* sbase = reinterpret_cast<const bf16*>(blk + size_t(total_rows) * row_bytes);
  const int iters = (rows + kOutIt - 1) / kOutIt;
  for (int it = 0; it < iters; ++it) {
    const int o = it * kOutIt + slot;
    const bool valid = ok && o < rows;
    float2 accA = f2(0.0f, 0.0f), accB = f2(0.0f, 0.0f);
    if (valid) {
      const unsigned char* wa = blk + size_t(o) * row_bytes;
      const unsigned char* wb = blk + size_t(o + rows) * row_bytes;
      const bf16* sa = sbase + o * groups;
      const bf16* sb = sbase + (o + rows) * groups;
      auto body = [&](int c) {
        float4 xv[kPlanes];
#pragma unroll
        for (int p = 0; p < kPlanes; ++p) xv[p] = sm.xs[p * chunks + c];
        const uint4 va = *reinterpret_cast<const uint4*>(wa + c * 16);
        uint4 vb;
        if constexpr (kPair) vb = *reinterpret_cast<const uint4*>(wb + c * 16);
        if constexpr (kW8) {
          float2 u = f2(0.0f, 0.0f), v = f2(0.0f, 0.0f);
          u = dot4_s8_x2(va.x, xv[0], u);
          v = dot4_s8_x2(va.y, xv[1], v);
          u = dot4_s8_x2(va.z, xv[2], u);
          v = dot4_s8_x2(va.w, xv[3], v);
          const float sc = __bfloat162float(sa[c >> 2]);
          accA = __ffma2_rn(u, f2(sc, sc), accA);
          accA = __ffma2_rn(v, f2(sc, sc), accA);
          if constexpr (kPair) {
            float2 u2 = f2(0.0f, 0.0f), v2 = f2(0.0f, 0.0f);
            u2 = dot4_s8_x2(vb.x, xv[0], u2);
            v2 = dot4_s8_x2(vb.y, xv[1], v2);
            u2 = dot4_s8_x2(vb.z, xv[2], u2);
            v2 = dot4_s8_x2(vb.w, xv[3], v2);
            const float sc2 = __bfloat162float(sb[c >> 2]);
            accB = __ffma2_rn(u2, f2(sc2, sc2), accB);
            accB = __ffma2_rn(v2, f2(sc2, sc2), accB);
          }
        } else {
          accA = dot4_bf16_x2(va.x, va.y, xv[0], accA);
          accA = dot4_bf16_x2(va.z, va.w, xv[1], accA);
          if constexpr (kPair) {
            accB = dot4_bf16_x2(vb.x, vb.y, xv[0], accB);
            accB = dot4_bf16_x2(vb.z, vb.w, xv[1], accB);
          }
        }
      };
      if constexpr (kK != 0) {
#pragma unroll
        for (int j = 0; j < kIt; ++j) {
          const int c = first + j * kSpan;
          if (kChunksK % kSpan == 0 || c < kChunksK) body(c);
        }
      } else {
#pragma unroll 2
        for (int c = first; c < chunks; c += kSpan) body(c);
      }
    }
    float vA = accA.x + accA.y, vB = accB.x + accB.y;
#pragma unroll
    for (int off = kLPR / 2; off > 0; off >>= 1) {
      vA += __shfl_xor_sync(0xffffffffu, vA, off);
      if constexpr (kPair) vB += __shfl_xor_sync(0xffffffffu, vB, off);
    }
    if constexpr (kWPR > 1) {
      float* part = sm.red_part + (cs.red_it & 1) * 2 * kPWarps;
      if (lane == 0) {
        part[cw] = vA;
        part[kPWarps + cw] = vB;
      }
      cbar();
      if (ksub == 0) {
        vA = 0.0f;
        vB = 0.0f;
#pragma unroll
        for (int j = 0; j < kWPR; ++j) {
          vA += part[cw + j];
          vB += part[kPWarps + cw + j];
        }
      }
    }
    ++cs.red_it;
    if (valid && ksub == 0 && ll == 0) epi(o, vA, vB);
  }
}

// Lane mapping per block: enough lanes per output to use the 16 warps in
// about one pass, compiled for the Qwen2.5-0.5B in_features (896 and 4864)
// and generic otherwise.
template <bool kW8, bool kPair, class Epi>
__device__ __forceinline__ void gemv_any(const unsigned char* blk, bool ok, int rows, int k,
                                         Consumer& cs, const Smem& sm, int ct, Epi epi) {
  if (k == 896) {
    if (rows > 32) {
      gemv_block<kW8, 896, 8, 1, kPair>(blk, ok, rows, k, cs, sm, ct, epi);
    } else if (rows > 16) {
      gemv_block<kW8, 896, 16, 1, kPair>(blk, ok, rows, k, cs, sm, ct, epi);
    } else {
      gemv_block<kW8, 896, 32, 2, kPair>(blk, ok, rows, k, cs, sm, ct, epi);
    }
  } else if (k == 4864 && !kPair) {
    gemv_block<kW8, 4864, 32, 2, kPair>(blk, ok, rows, k, cs, sm, ct, epi);
  } else if (rows > 8) {
    gemv_block<kW8, 0, 32, 1, kPair>(blk, ok, rows, k, cs, sm, ct, epi);
  } else if (rows > 4) {
    gemv_block<kW8, 0, 32, 2, kPair>(blk, ok, rows, k, cs, sm, ct, epi);
  } else if (rows > 2) {
    gemv_block<kW8, 0, 32, 4, kPair>(blk, ok, rows, k, cs, sm, ct, epi);
  } else {
    gemv_block<kW8, 0, 32, 8, kPair>(blk, ok, rows, k, cs, sm, ct, epi);
  }
}

// Attention of head blockIdx.x for the token at `pos` of layer `l`, with
// RoPE (half-split pairs, frequency theta^(-2i/64)) of q and k and the
// cache store of k / v at `pos` by the first head of each KV group.  Same
// arithmetic as attend_row (attention.cuh), FP32 partial sums in another
// order.
constexpr int kVPre = 8;  // V rows per warp loaded before the scores
__device__ __forceinline__ void trace_mark(const PersistArgs& a, int phase, int which, int ct) {
  if (a.trace != nullptr && ct == 0 && phase < a.trace_count) {
    a.trace[(size_t(blockIdx.x) * a.trace_count + phase) * 4 + which] = global_timer_ns();
  }
}

__device__ __forceinline__ bool attention_phase(const PersistArgs& a, const Smem& sm,
                                                const u64* qkv, u64* att, unsigned tag, int l,
                                                int pos, int ct, int phase) {
  constexpr int NW = kPWarps;
  constexpr int half = kHeadDim / 2;
  const int h = blockIdx.x;
  const int group = a.heads / a.kv_heads;
  const int kvh = h / group;
  const int lane = ct & 31, warp = ct >> 5;
  const int seq = pos + 1;
  float* qs = reinterpret_cast<float*>(sm.xs);
  float* kcur = qs + kHeadDim;
  float* vcur = kcur + kHeadDim;
  float* scores = vcur + kHeadDim;
  float* red = scores + seq;
  float* part = red + NW;
  const size_t cache_off = (size_t(l) * a.kv_heads + kvh) * a.max_seq * kHeadDim;
  bf16* kc = a.kcache + cache_off;
  bf16* vc = a.vcache + cache_off;
  const bool writer = h % group == 0;
  const uint32_t* vrow = reinterpret_cast<const uint32_t*>(vc) + lane;
  // 2. this step's q, k (rotated) and v
  float r0 = 0.0f, r1 = 0.0f;
  if (ct < 2 * half) {
    const int i = ct % half;
    const bool is_k = ct >= half;
    const int base = is_k ? (a.heads + kvh) * kHeadDim : h * kHeadDim;
    const float freq = powf(a.theta, -2.0f * float(i) / float(kHeadDim));
    float sn, cs;
    sincosf(float(pos) * freq, &sn, &cs);
    u64 w0 = 0, w1 = 0;
    wait_word2(qkv + base + i, qkv + base + i + half, tag, w0, w1, a, sm);
    trace_mark(a, phase, 3, ct);
    const float x0 = bf16_lo(lo16(w0)), x1 = bf16_lo(lo16(w1));
    r0 = bf16_round(x0 * cs - x1 * sn);
    r1 = bf16_round(x1 * cs + x0 * sn);
  } else if (ct < 2 * half + kHeadDim) {
    const int d = ct - 2 * half;
    u64 w = 0;
    wait_word(qkv + (a.heads + a.kv_heads + kvh) * kHeadDim + d, tag, w, a, sm);
    r0 = bf16_lo(lo16(w));
  }
  cbar();  // every warp is done with the previous phase's use of the region
  if (ct < 2 * half) {
    const int i = ct % half;
    float* dst = ct >= half ? kcur : qs;
    dst[i] = r0;
    dst[i + half] = r1;
  } else if (ct < 2 * half + kHeadDim) {
    vcur[ct - 2 * half] = r0;
  }
  if (cbar_or(*sm.abort_flag != 0)) return false;
  trace_mark(a, phase, 0, ct);
  // The first V rows of this warp, loaded before the scores are computed.
  uint32_t vr[kVPre];
#pragma unroll
  for (int j = 0; j < kVPre; ++j) {
    const int p = warp + j * NW;
    vr[j] = p < pos ? __ldcg(vrow + size_t(p) * half) : 0u;
  }
  // 3. scores (q as float4 broadcasts, four independent partial sums),
  //    softmax
  const float scale = rsqrtf(float(kHeadDim));
  const float4* q4 = reinterpret_cast<const float4*>(qs);
  float mx = -FLT_MAX;
  for (int p = ct; p < seq; p += kPConsumers) {
    float2 d0 = f2(0.0f, 0.0f), d1 = f2(0.0f, 0.0f);
    if (p == pos) {
      const float4* k4 = reinterpret_cast<const float4*>(kcur);
#pragma unroll
      for (int c = 0; c < kHeadDim / 4; ++c) {
        const float4 q = q4[c], kk = k4[c];
        d0 = __ffma2_rn(f2(q.x, q.y), f2(kk.x, kk.y), d0);
        d1 = __ffma2_rn(f2(q.z, q.w), f2(kk.z, kk.w), d1);
      }
    } else {
      uint4 w[8];
      const uint4* r = reinterpret_cast<const uint4*>(kc + size_t(p) * kHeadDim);
#pragma unroll
      for (int c = 0; c < 8; ++c) w[c] = __ldcg(r + c);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const float4 qa = q4[2 * c], qb = q4[2 * c + 1];
        d0 = __ffma2_rn(f2(qa.x, qa.y), f2(bf16_lo(w[c].x), bf16_hi(w[c].x)), d0);
        d1 = __ffma2_rn(f2(qa.z, qa.w), f2(bf16_lo(w[c].y), bf16_hi(w[c].y)), d1);
        d0 = __ffma2_rn(f2(qb.x, qb.y), f2(bf16_lo(w[c].z), bf16_hi(w[c].z)), d0);
        d1 = __ffma2_rn(f2(qb.z, qb.w), f2(bf16_lo(w[c].w), bf16_hi(w[c].w)), d1);
      }
    }
    const float sc = ((d0.x + d0.y) + (d1.x + d1.y)) * scale;
    scores[p] = sc;
    mx = fmaxf(mx, sc);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  if (lane == 0) red[warp] = mx;
  cbar();
  mx = red[0];
#pragma unroll
  for (int w = 1; w < NW; ++w) mx = fmaxf(mx, red[w]);
  cbar();
  float sum = 0.0f;
  for (int p = ct; p < seq; p += kPConsumers) {
    const float e = expf(scores[p] - mx);
    scores[p] = e;
    sum += e;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
  if (lane == 0) red[warp] = sum;
  cbar();
  // 4. P.V: warp w takes positions w, w + 16, ...; lane l dims 2l, 2l + 1
  //    (two independent accumulator pairs)
  float2 acc0 = f2(0.0f, 0.0f), acc1 = f2(0.0f, 0.0f);
#pragma unroll
  for (int j = 0; j < kVPre; ++j) {
    const int p = warp + j * NW;
    if (p < seq) {
      const float pr = scores[p];
      const float2 v = p == pos ? f2(vcur[2 * lane], vcur[2 * lane + 1])
                                : f2(bf16_lo(vr[j]), bf16_hi(vr[j]));
      if (j & 1) {
        acc1 = __ffma2_rn(f2(pr, pr), v, acc1);
      } else {
        acc0 = __ffma2_rn(f2(pr, pr), v, acc0);
      }
    }
  }
  for (int p = warp + kVPre * NW; p < seq; p += NW) {
    const float pr = scores[p];
    float2 v;
    if (p == pos) {
      v = f2(vcur[2 * lane], vcur[2 * lane + 1]);
    } else {
      const uint32_t raw = __ldcg(vrow + size_t(p) * half);
      v = f2(bf16_lo(raw), bf16_hi(raw));
    }
    acc0 = __ffma2_rn(f2(pr, pr), v, acc0);
  }
  const float a0 = acc0.x + acc1.x, a1 = acc0.y + acc1.y;
  part[warp * kHeadDim + 2 * lane] = a0;
  part[warp * kHeadDim + 2 * lane + 1] = a1;
  cbar();
  trace_mark(a, phase, 2, ct);
  if (ct < kHeadDim) {
    float denom = 0.0f, o = 0.0f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      denom += red[w];
      o += part[w * kHeadDim + ct];
    }
    st_word(att + h * kHeadDim + ct, tag_word(__float2bfloat16_rn(o / denom), tag));
  }
  // The new position's k / v into the cache (read from the next step on).
  // The storing threads fence at the start of the next stage, while they
  // wait for its input anyway: that orders the stores before every later
  // output of this CTA, and so before every read of them.
  if (writer && ct < 2 * kHeadDim) {
    const float v = ct < kHeadDim ? kcur[ct] : vcur[ct - kHeadDim];
    bf16* dst = ct < kHeadDim ? kc : vc;
    dst[size_t(pos) * kHeadDim + (ct & (kHeadDim - 1))] = __float2bfloat16_rn(v);
  }
  return true;
}

template <bool kW8>
__global__ void __launch_bounds__(kPThreads, 1) decode_persistent_kernel(const PersistArgs a) {
  extern __shared__ __align__(128) unsigned char psmem[];
  Smem sm;
  sm.ring = psmem;
  sm.xs = reinterpret_cast<float4*>(psmem + a.region_off);
  uint64_t* bars = reinterpret_cast<uint64_t*>(psmem + a.bars_off);
  sm.bar_full = smem_u32(bars);
  sm.bar_empty = sm.bar_full + 8 * kNDesc;
  int* misc = reinterpret_cast<int*>(bars + 2 * kNDesc);
  sm.desc_off = misc;
  sm.abort_flag = misc + kNDesc;
  sm.s_issued = misc + kNDesc + 1;
  sm.s_consumed = misc + kNDesc + 2;
  sm.red_v = reinterpret_cast<float*>(misc + kNDesc + 4);
  sm.red_i = misc + kNDesc + 4 + kPWarps;
  sm.red_part = reinterpret_cast<float*>(misc + kNDesc + 4 + 2 * kPWarps);
  sm.norm_red = sm.red_part + 4 * kPWarps;
  sm.bias_s = sm.norm_red + kPWarps;
  sm.x_layer = reinterpret_cast<bf16*>(psmem + a.raw_off);
  sm.x_mid = sm.x_layer + a.hidden;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int d = 0; d < kNDesc; ++d) {
      mbar_init(sm.bar_full + 8 * d, 1);
      mbar_init(sm.bar_empty + 8 * d, kPWarps);
    }
    *sm.abort_flag = 0;
    *sm.s_issued = 0;
    *sm.s_consumed = INT_MAX;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  const int qkv_dim = (a.heads + 2 * a.kv_heads) * kHeadDim;
  const size_t layer_words = persist_layer_words(qkv_dim, a.hidden, a.inter);
  const int lm_tiles = (a.vocab + a.lm_rows - 1) / a.lm_rows;

  if (warp == 0) {
    if (lane == 0) {
      Producer pr;
      bool ok = true;
      for (int step = 0; step < a.steps && ok; ++step) {
        for (int l = 0; l < a.n_layers && ok; ++l) {
          const PersistLayer L = a.layers[l];
          for (int role = kRoleQkv; role <= kRoleDown && ok; ++role) {
            for (int t = 0; t < a.subs[role] && ok; ++t) {
              ok = produce(block_of(a, L, role, kW8, t), pr, sm, a);
            }
          }
        }
        for (int t = blockIdx.x; t < lm_tiles && ok; t += gridDim.x) {
          ok = produce(block_of(a, a.layers[0], kRoleLm, false, t), pr, sm, a);
        }
      }
      *sm.s_issued = pr.j;
    }
  } else {
    const int ct = threadIdx.x - 32;
    const int cw = ct >> 5;
    const int H = a.hidden;
    const int pos0 = *a.d_pos;
    const int step0 = *a.d_step;
    int tok = *a.d_token;
    Consumer cs;
    bool alive = true;
    int phase = 0;
    auto mark = [&](int which) {
      if (a.trace != nullptr && ct == 0 && phase < a.trace_count) {
        a.trace[(size_t(blockIdx.x) * a.trace_count + phase) * 4 + which] = global_timer_ns();
      }
    };
    u64* partials = a.words + size_t(a.n_layers) * layer_words;
    for (int step = 0; step < a.steps && alive; ++step) {
      const int pos = pos0 + step;
      const unsigned tag = a.epoch + unsigned(step) + 1u;
      const bf16* emb = a.embed + size_t(tok) * H;  // x entering layer 0
      const u64* x_in = nullptr;                     // x entering layer l (tagged)
      for (int l = 0; l < a.n_layers; ++l) {
        if (a.stall_phase >= 0 && blockIdx.x == 0 && step == 0 && phase >= a.stall_phase) {
          alive = false;  // test hook: the other CTAs' waits for this CTA expire
          break;
        }
        const PersistLayer L = a.layers[l];
        u64* w_qkv = a.words + size_t(l) * layer_words;
        u64* w_att = w_qkv + qkv_dim;
        u64* w_xo = w_att + H;
        u64* w_h = w_xo + H;
        u64* w_xd = w_h + a.inter;
        // ---- q | k | v = W_qkv RMSNorm(x) + b
        {
          const int share0 = int(blockIdx.x) * a.rows[kRoleQkv];
          if (ct < a.rows[kRoleQkv] && share0 + ct < qkv_dim) {
            sm.bias_s[ct] = L.qkv_b ? __bfloat162float(L.qkv_b[share0 + ct]) : 0.0f;
          }
        }
        if (!(alive = stage<kW8 ? 16 : 8>(x_in, emb, tag, H, L.in_norm, a.eps, sm.x_layer, a,
                                          sm, ct, phase))) {
          break;
        }
        mark(0);
        {
          for (int t = 0; t < a.subs[kRoleQkv]; ++t) {
            const Block b = block_of(a, L, kRoleQkv, kW8, t);
            if (b.rows == 0) continue;
            const unsigned char* blk;
            const bool ok = acquire(cs, sm, a, blk);
            mark(2);
            gemv_any<kW8, false>(blk, ok, b.rows, b.k, cs, sm, ct, [&](int o, float v, float) {
              const int row = b.row0 + o;
              const float bias = sm.bias_s[row - int(blockIdx.x) * a.rows[kRoleQkv]];
              st_word(w_qkv + row, tag_word(__float2bfloat16_rn(v + bias), tag));
            });
            release(cs, sm, ok, lane);
          }
        }
        mark(1);
        ++phase;
        // ---- attention (CTA h: head h)
        if (int(blockIdx.x) < a.heads) {
          if (!(alive = attention_phase(a, sm, w_qkv, w_att, tag, l, pos, ct, phase))) break;
        }
        mark(1);
        ++phase;
        // ---- x += W_o att
        if (int(blockIdx.x) < a.heads && int(blockIdx.x) % (a.heads / a.kv_heads) == 0 &&
            ct < 2 * kHeadDim) {
          __threadfence();  // KV-cache stores of the attention phase
        }
        if (!(alive = stage<kW8 ? 16 : 8>(w_att, nullptr, tag, H, nullptr, 0.0f, nullptr, a, sm,
                                          ct, phase))) {
          break;
        }
        mark(0);
        {
          for (int t = 0; t < a.subs[kRoleO]; ++t) {
            const Block b = block_of(a, L, kRoleO, kW8, t);
            if (b.rows == 0) continue;
            const unsigned char* blk;
            const bool ok = acquire(cs, sm, a, blk);
            mark(2);
            gemv_any<kW8, false>(blk, ok, b.rows, b.k, cs, sm, ct, [&](int o, float v, float) {
              const int row = b.row0 + o;
              const float xr = __bfloat162float(sm.x_layer[row]);
              const float y = bf16_round(v);
              st_word(w_xo + row, tag_word(__float2bfloat16_rn(xr + y), tag));
            });
            release(cs, sm, ok, lane);
          }
        }
        mark(1);
        ++phase;
        // ---- h = silu(gate) * up, [gate; up] = W_gu RMSNorm(x)
        if (!(alive = stage<kW8 ? 16 : 8>(w_xo, nullptr, tag, H, L.post_norm, a.eps, sm.x_mid, a, sm,
                                          ct, phase))) {
          break;
        }
        mark(0);
        {
          for (int t = 0; t < a.subs[kRoleGateUp]; ++t) {
            const Block b = block_of(a, L, kRoleGateUp, kW8, t);
            if (b.rows == 0) continue;
            const unsigned char* blk;
            const bool ok = acquire(cs, sm, a, blk);
            mark(2);
            gemv_any<kW8, true>(blk, ok, b.rows, b.k, cs, sm, ct, [&](int o, float g, float u) {
              const float gv = bf16_round(g), uv = bf16_round(u);
              const float hv = gv / (1.0f + expf(-gv)) * uv;
              st_word(w_h + b.row0 + o, tag_word(__float2bfloat16_rn(hv), tag));
            });
            release(cs, sm, ok, lane);
          }
        }
        mark(1);
        ++phase;
        // ---- x += W_down h
        if (!(alive = stage<kW8 ? 16 : 8>(w_h, nullptr, tag, a.inter, nullptr, 0.0f, nullptr, a, sm,
                                          ct, phase))) {
          break;
        }
        mark(0);
        {
          for (int t = 0; t < a.subs[kRoleDown]; ++t) {
            const Block b = block_of(a, L, kRoleDown, kW8, t);
            if (b.rows == 0) continue;
            const unsigned char* blk;
            const bool ok = acquire(cs, sm, a, blk);
            mark(2);
            gemv_any<kW8, false>(blk, ok, b.rows, b.k, cs, sm, ct, [&](int o, float v, float) {
              const int row = b.row0 + o;
              const float xr = __bfloat162float(sm.x_mid[row]);
              const float y = bf16_round(v);
              st_word(w_xd + row, tag_word(__float2bfloat16_rn(xr + y), tag));
            });
            release(cs, sm, ok, lane);
          }
        }
        mark(1);
        ++phase;
        x_in = w_xd;
      }
      if (!alive) break;
      // ---- logits = E RMSNorm(x); per-CTA argmax partial
      if (!(alive = stage<8>(x_in, emb, tag, H, a.final_norm, a.eps, nullptr, a, sm, ct, phase))) break;
      mark(0);
      float best = -FLT_MAX;
      int best_index = INT_MAX;
      for (int t = blockIdx.x; t < lm_tiles; t += gridDim.x) {
        const Block b = block_of(a, a.layers[0], kRoleLm, false, t);
        const unsigned char* blk;
        const bool ok = acquire(cs, sm, a, blk);
        if (t == int(blockIdx.x)) mark(2);
        gemv_any<false, false>(blk, ok, b.rows, b.k, cs, sm, ct, [&](int o, float v, float) {
          const int row = b.row0 + o;
          const bf16 y = __float2bfloat16_rn(v);
          a.logits[row] = y;
          argmax_update(best, best_index, __bfloat162float(y), row);
        });
        release(cs, sm, ok, lane);
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, off);
        const int oi = __shfl_xor_sync(0xffffffffu, best_index, off);
        argmax_update(best, best_index, ov, oi);
      }
      if (lane == 0) {
        sm.red_v[cw] = best;
        sm.red_i[cw] = best_index;
      }
      cbar();
      if (ct == 0) {
        float b = -FLT_MAX;
        int bi = INT_MAX;
        for (int w = 0; w < kPWarps; ++w) argmax_update(b, bi, sm.red_v[w], sm.red_i[w]);
        st_word(partials + blockIdx.x, (u64(tag) << 32) | u64(__float_as_uint(b)));
        st_word(partials + gridDim.x + blockIdx.x, (u64(tag) << 32) | u64(uint32_t(bi)));
      }
      cbar();  // red_v / red_i read by consumer thread 0 before they are reused
      mark(1);
      ++phase;
      // ---- next token: argmax over the CTAs' partials
      float b = -FLT_MAX;
      int bi = INT_MAX;
      for (int j = ct; j < int(gridDim.x); j += kPConsumers) {
        u64 wv = 0, wi = 0;
        wait_word(partials + j, tag, wv, a, sm);
        wait_word(partials + gridDim.x + j, tag, wi, a, sm);
        argmax_update(b, bi, __uint_as_float(uint32_t(wv)), int(uint32_t(wi)));
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, b, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        argmax_update(b, bi, ov, oi);
      }
      if (lane == 0) {
        sm.red_v[cw] = b;
        sm.red_i[cw] = bi;
      }
      if (cbar_or(*sm.abort_flag != 0)) {
        alive = false;
        break;
      }
      b = -FLT_MAX;
      bi = INT_MAX;
      for (int w = 0; w < kPWarps; ++w) argmax_update(b, bi, sm.red_v[w], sm.red_i[w]);
      tok = bi == INT_MAX ? 0 : bi;
      if (blockIdx.x == 0 && ct == 0 && step0 + step < a.max_out) a.d_out[step0 + step] = tok;
      cbar();  // red_v / red_i reusable
      mark(0);
      mark(1);
      ++phase;
    }
    if (lane == 0) atomicMin(sm.s_consumed, cs.fail >= 0 ? cs.fail : cs.j);
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
  // this CTA's ring before the CTA exits (blocks are reissued only after all
  // consumer warps saw the previous copy of their descriptor land).
  if (threadIdx.x == 0) {
    for (int j = *sm.s_consumed; j < *sm.s_issued; ++j) {
      const int d = j % kNDesc;
      const uint32_t parity = uint32_t(j / kNDesc) & 1u;
      const uint64_t start = global_timer_ns();
      while (!mbar_try_wait(sm.bar_full + 8 * d, parity)) {
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

int gcd(int a, int b) { return b == 0 ? a : gcd(b, a % b); }

// Rows per CTA for an n-row matrix of in_features k: ceil(n / grid),
// rounded up so that every block's scale rows start on 16 bytes.
int rows_per_cta(int n, int k, bool w8, int grid) {
  const int align = w8 ? 8 / gcd(k / 64, 8) : 1;
  const int per = (n + grid - 1) / grid;
  return (per + align - 1) / align * align;
}

}  // namespace

PersistPlan plan_persistent(bool w8, int hidden, int inter, int heads, int kv_heads, int vocab,
                            int max_seq) {
  PersistPlan p;
  if (hidden % 64 != 0 || inter % 64 != 0 || hidden > kPMaxStageK || inter > kPMaxStageK ||
      heads * kHeadDim != hidden || heads % kv_heads != 0 || max_seq <= 0 || vocab % 8 != 0) {
    return p;
  }
  const int grid = sm_count();
  if (heads > grid) return p;
  const int qkv_dim = (heads + 2 * kv_heads) * kHeadDim;
  p.rows[kRoleQkv] = rows_per_cta(qkv_dim, hidden, w8, grid);
  p.rows[kRoleO] = rows_per_cta(hidden, hidden, w8, grid);
  p.rows[kRoleGateUp] = rows_per_cta(inter, hidden, w8, grid);
  p.rows[kRoleDown] = rows_per_cta(hidden, inter, w8, grid);
  const size_t stage_bytes = size_t(hidden > inter ? hidden : inter) * 4;
  const size_t att_bytes = (attend_smem_floats<kPConsumers>(max_seq) + 3 * kHeadDim) * 4;
  const int scratch = int(((stage_bytes > att_bytes ? stage_bytes : att_bytes) + 127) / 128 * 128);
  const int region = scratch + (4 * hidden + 127) / 128 * 128;  // + x_layer, x_mid
  const int bars = 16 * kNDesc;
  const int ring = (kPSmemLimit - region - bars - kPMisc) / 128 * 128;
  if (ring <= 0) return p;
  auto bytes = [&](int rows, int k, bool q, int parts) {
    return size_t(parts) * rows * ((q ? size_t(k) : 2 * size_t(k)) + (q ? size_t(k / 64) * 2 : 0));
  };
  // A CTA's share is streamed as blocks of at most a third of the ring.
  const int ks[4] = {hidden, hidden, hidden, inter};
  for (int r = 0; r < 4; ++r) {
    const int parts = r == kRoleGateUp ? 2 : 1;
    const int align = w8 ? 8 / gcd(ks[r] / 64, 8) : 1;
    int sub = p.rows[r];
    while (sub > align && bytes(sub, ks[r], w8, parts) > size_t(ring) / 3) sub -= align;
    if (bytes(sub, ks[r], w8, parts) > size_t(ring) / 3) return p;
    p.sub_rows[r] = sub;
    p.subs[r] = (p.rows[r] + sub - 1) / sub;
  }
  p.lm_rows = 0;
  for (int r : {32, 16, 8}) {
    if (bytes(r, hidden, false, 1) <= size_t(ring) / 3) {
      p.lm_rows = r;
      break;
    }
  }
  if (p.lm_rows == 0) return p;
  if (p.rows[kRoleQkv] > kPMaxBias) return p;
  p.ring_bytes = ring;
  p.region_off = ring;
  p.raw_off = ring + scratch;
  p.bars_off = ring + region;
  p.smem = p.bars_off + bars + kPMisc;
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
  a.ring_bytes = plan.ring_bytes;
  a.region_off = plan.region_off;
  a.raw_off = plan.raw_off;
  a.bars_off = plan.bars_off;
  for (int r = 0; r < 4; ++r) {
    a.rows[r] = plan.rows[r];
    a.sub_rows[r] = plan.sub_rows[r];
    a.subs[r] = plan.subs[r];
  }
  a.lm_rows = plan.lm_rows;
  cudaError_t e = cudaMemsetAsync(a.grid_abort, 0, sizeof(int), stream);
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
