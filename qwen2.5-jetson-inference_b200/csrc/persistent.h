// Internal interface of the persistent decode kernel (decode_persistent.cu)
// for the engine (engine.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>

namespace b200 {

using bf16 = __nv_bfloat16;

// One layer's weights as the kernel reads them (device copy of the array).
// gu_w holds the gate rows followed by the up rows ([gate; up]).
struct PersistLayer {
  const void* qkv_w;
  const bf16* qkv_s;
  const bf16* qkv_b;
  const void* o_w;
  const bf16* o_s;
  const void* gu_w;
  const bf16* gu_s;
  const void* down_w;
  const bf16* down_s;
  const bf16* in_norm;
  const bf16* post_norm;
};

// Matrix roles of a decode step, in stream order.
enum PersistRole { kRoleQkv = 0, kRoleO = 1, kRoleGateUp = 2, kRoleDown = 3, kRoleLm = 4 };

// Tagged activation words (64 bit: BF16 value bits in the low half, the
// step's tag in the high half) of one layer: qkv, attention output, x after
// o_proj, silu(gate) * up, x after down_proj.
__host__ __device__ constexpr size_t persist_layer_words(int qkv_dim, int hidden, int inter) {
  return size_t(qkv_dim) + 3 * size_t(hidden) + size_t(inter);
}
// Whole tagged buffer: layers x layer words + 2 words per CTA (LM-head
// argmax partials: value, index).
__host__ __device__ constexpr size_t persist_words(int layers, int qkv_dim, int hidden,
                                                   int inter, int grid) {
  return size_t(layers) * persist_layer_words(qkv_dim, hidden, inter) + 2 * size_t(grid);
}

struct PersistArgs {
  const PersistLayer* layers;
  int n_layers;
  int hidden, inter, heads, kv_heads, vocab, max_seq;
  float eps, theta;
  const bf16* embed;           // [vocab, hidden], also the tied LM head
  const bf16* final_norm;
  unsigned long long* words;   // tagged activations (persist_words), zeroed at creation
  unsigned epoch;              // tag of step s is epoch + s + 1
  bf16* logits;                // [vocab]
  bf16* kcache;                // [layers][kv_heads][max_seq][64]
  bf16* vcache;
  int* d_token;
  int* d_pos;
  int* d_step;
  int* d_out;
  int max_out;
  int* grid_abort;             // zeroed before each launch
  int* status;                 // first B200_DEVICE_* error, sticky
  // Optional timeline (nullptr: off): for the first trace_count phases of
  // the launch, [cta][phase][input staged, phase done, first weight block
  // landed, input words arrived] global-timer ns.
  unsigned long long* trace;
  int trace_count;
  // Test hook (-1: off): CTA 0 stops before layer phase `stall_phase` of the
  // first step, so every other CTA's bounded wait for its outputs expires.
  int stall_phase;
  int steps;
  // plan (copied from PersistPlan by launch_persistent)
  int ring_bytes;              // shared memory: weight ring at 0, staging
  int region_off;              // region at region_off (x copies at raw_off),
  int raw_off;                 // barriers and block descriptors at bars_off
  int bars_off;
  int rows[4];                 // share per CTA (rows; gate|up: row pairs), by role
  int sub_rows[4];             // rows per block of a share
  int subs[4];                 // blocks per share
  int lm_rows;                 // rows per LM-head tile
};

struct PersistPlan {
  bool ok = false;
  int grid = 0;
  int smem = 0;
  int ring_bytes = 0;
  int region_off = 0;
  int raw_off = 0;
  int bars_off = 0;
  int rows[4] = {0, 0, 0, 0};
  int sub_rows[4] = {0, 0, 0, 0};
  int subs[4] = {0, 0, 0, 0};
  int lm_rows = 0;
};

// Plans the kernel for the shapes (ok == false: shapes it does not take).
PersistPlan plan_persistent(bool w8, int hidden, int inter, int heads, int kv_heads,
                            int vocab, int max_seq);
// Cooperative launch of `a.steps` decode steps on `stream`.
cudaError_t launch_persistent(bool w8, const PersistPlan& plan, const PersistArgs& a,
                              cudaStream_t stream);

}  // namespace b200
