// Internal interface of the persistent decode kernel (decode_persistent.cu)
// for the engine (engine.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace b200 {

using bf16 = __nv_bfloat16;

// One layer's weights as the kernel reads them (device copy of the array).
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

struct PersistArgs {
  const PersistLayer* layers;
  int n_layers;
  int hidden, inter, heads, kv_heads, vocab, max_seq;
  float eps, theta;
  const bf16* embed;       // [vocab, hidden], also the tied LM head
  const bf16* final_norm;
  bf16* x;                 // [hidden] residual stream
  bf16* qkv;               // [(heads + 2 kv_heads) * 64]
  bf16* att;               // [hidden]
  bf16* gu;                // [2 * inter]
  bf16* logits;            // [vocab]
  bf16* kcache;            // [layers][kv_heads][max_seq][64]
  bf16* vcache;
  float* part_v;           // [grid] LM-head argmax partials
  int* part_i;
  int* d_token;
  int* d_pos;
  int* d_step;
  int* d_out;
  int max_out;
  unsigned* grid_counter;  // zeroed before each launch
  int* grid_abort;         // zeroed before each launch
  int* status;             // first B200_DEVICE_* error, sticky
  // Optional timeline (nullptr: off): for the first trace_count grid
  // barriers, [cta][barrier][arrive, leave] global-timer nanoseconds.
  unsigned long long* trace;
  int trace_count;
  int steps;
  int stages;
  int slot_bytes;
  int region_off;          // shared-memory layout (bytes): ring at 0, then
  int bars_off;            // the staging / attention region, then barriers
  int rpt[5];              // rows per tile of each role
};

struct PersistPlan {
  bool ok = false;
  int grid = 0;
  int smem = 0;
  int stages = 0;
  int slot_bytes = 0;
  int region_off = 0;
  int bars_off = 0;
  int rpt[5] = {0, 0, 0, 0, 0};
};

// Plans the kernel for the shapes (ok == false: shapes it does not take).
PersistPlan plan_persistent(bool w8, int hidden, int inter, int heads, int kv_heads,
                            int vocab, int max_seq);
// Cooperative launch of `a.steps` decode steps on `stream`.
cudaError_t launch_persistent(bool w8, const PersistPlan& plan, const PersistArgs& a,
                              cudaStream_t stream);

}  // namespace b200
