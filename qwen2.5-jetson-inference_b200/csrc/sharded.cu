// Column-sharded Linear across the GPUs of one node (one process per GPU):
//
//  * W8A16 GEMM: rank r owns weight rows (= output columns)
//    [r*N/P, (r+1)*N/P) and their scales; X is replicated.  The local
//    tensor-core GEMM writes Y_r [M, N/P] straight into slot r of a gather
//    buffer [P][M][N/P], an in-place ncclAllGather fills the other slots over
//    NVLink, and a copy kernel lays the slots out as the row-major [M, N]
//    output the engine expects.
//    The fused form (b200_sharded_gemm_w8a16_p2p) has no NCCL data path: the
//    GEMM epilogue stores every output tile into the window buffer of every
//    rank (CUDA IPC mappings, 16-byte stores over NVLink), at its final
//    [M, N] position, while the next tiles are computed.
//  * LM head: rank r owns vocabulary rows [r*V/P, (r+1)*V/P).  The local
//    fused GEMV + argmax yields (BF16 logit, global index); it is packed into
//    a 64-bit key that orders by value and then by lower index,
//    (orderable(value) << 32) | (0xFFFFFFFF - index), so the largest of the
//    P keys is the global argmax with the reference's lowest-index tie rule
//    (src/cuda/kernels.cu:545-603).  With P > 1 one kernel per rank stores
//    its key into every rank's slot window over NVLink and reduces the P
//    keys of its own window (no collective call).
//
// The reference has no multi-GPU path; these are the sharded forms of its
// gemm_w8a16 and lm_head_bf16 (src/cuda/kernels.cu:1566-1579, 1657-1684).
#include <nccl.h>

#include <cfloat>
#include <climits>
#include <cstring>
#include <new>
#include <vector>

#include "b200_linear.h"
#include "common.cuh"
#include "kernels.h"

struct b200_window;

struct b200_comm {
  ncclComm_t nccl = nullptr;
  int nranks = 1;
  int rank = 0;
  bool owned = false;
  b200_window* keys = nullptr;  // argmax exchange slots (created on first use)
  unsigned long long seq = 0;   // exchanges so far (same on every rank)
};

struct b200_window {
  void* local = nullptr;
  size_t bytes = 0;
  int nranks = 1;
  int rank = 0;
  void* peer[8] = {};  // peer[r]: rank r's buffer in this process
  int* token = nullptr;  // 4-byte operand of the ordering all-reduce
};

namespace b200 {

constexpr int kMaxRanks = 8;  // ranks of one node (windows map at most 8)

namespace {

// [P][M][Ns] -> [M][P*Ns], 16 bytes per thread per step.
__global__ void __launch_bounds__(256)
gather_to_rows_kernel(const uint4* __restrict__ slots, uint4* __restrict__ out,
                      int nranks, int m, int ns_vec) {
  const size_t per_slot = size_t(m) * ns_vec;
  const size_t total = per_slot * nranks;
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < total;
       i += size_t(gridDim.x) * blockDim.x) {
    const size_t r = i / per_slot;
    const size_t rem = i - r * per_slot;
    const size_t row = rem / ns_vec;
    const size_t c = rem - row * ns_vec;
    out[row * (size_t(ns_vec) * nranks) + r * ns_vec + c] = slots[i];
  }
}

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && v > -FLT_MAX && i < bi);
}

// Reduces the local per-CTA partials to one packed key with a global index.
__global__ void __launch_bounds__(1024)
local_argmax_key_kernel(const float* __restrict__ block_value,
                        const int* __restrict__ block_index, int count,
                        int index_offset, unsigned long long* __restrict__ key) {
  __shared__ float sv[32];
  __shared__ int si[32];
  pdl_wait_primary();
  float best = -FLT_MAX;
  int best_index = INT_MAX;
  for (int i = threadIdx.x; i < count; i += blockDim.x) {
    if (better(block_value[i], block_index[i], best, best_index)) {
      best = block_value[i];
      best_index = block_index[i];
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, off);
    const int oi = __shfl_xor_sync(0xffffffffu, best_index, off);
    if (better(ov, oi, best, best_index)) {
      best = ov;
      best_index = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = best;
    si[threadIdx.x >> 5] = best_index;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = -FLT_MAX;
    int bi = INT_MAX;
    for (int w = 0; w < int(blockDim.x >> 5); ++w) {
      if (better(sv[w], si[w], b, bi)) {
        b = sv[w];
        bi = si[w];
      }
    }
    // No value above -FLT_MAX on this shard: key 0 loses to every real one
    // (and decodes to index 0 if all shards are empty, as argmax_bf16 does).
    unsigned long long k = 0ull;
    if (bi != INT_MAX) {
      const unsigned int gi = unsigned(bi + index_offset);
      k = (static_cast<unsigned long long>(float_order_key(b)) << 32) |
          (0xFFFFFFFFull - gi);
    }
    *key = k;
  }
}

__global__ void decode_argmax_key_kernel(const unsigned long long* __restrict__ key,
                                         int* __restrict__ argmax) {
  const unsigned long long k = *key;
  *argmax = k == 0ull ? 0 : int(0xFFFFFFFFull - (k & 0xFFFFFFFFull));
}

__device__ int g_comm_status = 0;

// Cross-GPU argmax without a collective: reduces this rank's per-CTA
// partials to a key, stores (key, seq) into slot `rank` of every rank's
// window (NVLink stores: key, system fence, then the sequence number), waits
// (bounded) until every slot of its own window carries `seq`, and decodes
// the largest key.  One CTA per rank; waits end after kWaitTimeoutNs with
// B200_DEVICE_TIMEOUT_GRID in g_comm_status.
struct KeySlots {
  unsigned long long* slot[8];  // rank q's window, as mapped in this process
};

__global__ void __launch_bounds__(256)
exchange_argmax_kernel(const float* __restrict__ block_value,
                       const int* __restrict__ block_index, int count, int index_offset,
                       KeySlots windows, int nranks, int rank, unsigned long long seq,
                       int* __restrict__ argmax) {
  __shared__ float sv[32];
  __shared__ int si[32];
  __shared__ unsigned long long keys[8];
  pdl_wait_primary();
  float best = -FLT_MAX;
  int best_index = INT_MAX;
  for (int i = threadIdx.x; i < count; i += blockDim.x) {
    if (better(block_value[i], block_index[i], best, best_index)) {
      best = block_value[i];
      best_index = block_index[i];
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, off);
    const int oi = __shfl_xor_sync(0xffffffffu, best_index, off);
    if (better(ov, oi, best, best_index)) {
      best = ov;
      best_index = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = best;
    si[threadIdx.x >> 5] = best_index;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = -FLT_MAX;
    int bi = INT_MAX;
    for (int w = 0; w < int(blockDim.x >> 5); ++w) {
      if (better(sv[w], si[w], b, bi)) {
        b = sv[w];
        bi = si[w];
      }
    }
    unsigned long long k = 0ull;
    if (bi != INT_MAX) {
      const unsigned int gi = unsigned(bi + index_offset);
      k = (static_cast<unsigned long long>(float_order_key(b)) << 32) | (0xFFFFFFFFull - gi);
    }
    // Slot layout per window: [seq parity][rank][key, seq].  Consecutive
    // calls use different halves, so a rank that is one call ahead never
    // overwrites a key that a slower rank has not read yet; it cannot get two
    // calls ahead, since finishing call seq+1 needs the slower rank's key of
    // call seq+1, published only after that rank has read call seq.
    const int half = int(seq & 1ull) * 2 * kMaxRanks;
    for (int q = 0; q < nranks; ++q) {
      volatile unsigned long long* dst = windows.slot[q] + half + 2 * rank;
      dst[0] = k;
    }
    __threadfence_system();
    for (int q = 0; q < nranks; ++q) {
      volatile unsigned long long* dst = windows.slot[q] + half + 2 * rank;
      dst[1] = seq;
    }
  }
  if (threadIdx.x < nranks) {
    const int half = int(seq & 1ull) * 2 * kMaxRanks;
    volatile unsigned long long* mine = windows.slot[rank] + half + 2 * threadIdx.x;
    const uint64_t start = global_timer_ns();
    unsigned long long k = 0ull;
    while (true) {
      if (mine[1] >= seq) {
        __threadfence_system();
        k = mine[0];
        break;
      }
      if (global_timer_ns() - start > kWaitTimeoutNs) {
        atomicCAS(&g_comm_status, 0, B200_DEVICE_TIMEOUT_GRID);
        break;
      }
    }
    keys[threadIdx.x] = k;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long k = 0ull;
    for (int q = 0; q < nranks; ++q) k = keys[q] > k ? keys[q] : k;
    *argmax = k == 0ull ? 0 : int(0xFFFFFFFFull - (k & 0xFFFFFFFFull));
  }
}

int nccl_status(ncclResult_t r) { return r == ncclSuccess ? B200_OK : B200_ERR_NCCL; }

}  // namespace

cudaError_t read_comm_status(int* value, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(value, g_comm_status, sizeof(int));
  if (e != cudaSuccess || !clear) return e;
  const int zero = 0;
  return cudaMemcpyToSymbol(g_comm_status, &zero, sizeof(int));
}

}  // namespace b200

using b200::bf16;

extern "C" {

int b200_nccl_unique_id_bytes(void) { return int(sizeof(ncclUniqueId)); }

int b200_nccl_get_unique_id(void* out) {
  if (out == nullptr) return B200_ERR_INVALID_ARGUMENT;
  ncclUniqueId id;
  if (ncclGetUniqueId(&id) != ncclSuccess) return B200_ERR_NCCL;
  memcpy(out, &id, sizeof(id));
  return B200_OK;
}

int b200_comm_init(b200_comm_t* comm, const void* unique_id, int nranks,
                   int rank) {
  if (comm == nullptr || unique_id == nullptr || nranks < 1 || rank < 0 ||
      rank >= nranks) {
    return B200_ERR_INVALID_ARGUMENT;
  }
  ncclUniqueId id;
  memcpy(&id, unique_id, sizeof(id));
  auto* c = new (std::nothrow) b200_comm;
  if (c == nullptr) return B200_ERR_INVALID_ARGUMENT;
  if (ncclCommInitRank(&c->nccl, nranks, id, rank) != ncclSuccess) {
    delete c;
    return B200_ERR_NCCL;
  }
  c->nranks = nranks;
  c->rank = rank;
  c->owned = true;
  *comm = c;
  return B200_OK;
}

int b200_comm_wrap(b200_comm_t* comm, void* nccl_comm, int nranks, int rank) {
  if (comm == nullptr || nccl_comm == nullptr || nranks < 1 || rank < 0 ||
      rank >= nranks) {
    return B200_ERR_INVALID_ARGUMENT;
  }
  auto* c = new (std::nothrow) b200_comm;
  if (c == nullptr) return B200_ERR_INVALID_ARGUMENT;
  c->nccl = static_cast<ncclComm_t>(nccl_comm);
  c->nranks = nranks;
  c->rank = rank;
  c->owned = false;
  *comm = c;
  return B200_OK;
}

int b200_comm_destroy(b200_comm_t comm) {
  if (comm == nullptr) return B200_OK;
  int rc = b200_window_destroy(comm->keys);
  comm->keys = nullptr;
  if (comm->owned && comm->nccl != nullptr) {
    const int r2 = b200::nccl_status(ncclCommDestroy(comm->nccl));
    if (rc == B200_OK) rc = r2;
  }
  delete comm;
  return rc;
}

int b200_window_create(b200_comm_t comm, size_t bytes, b200_stream_t stream,
                       b200_window_t* out) {
  if (comm == nullptr || out == nullptr || bytes == 0 || comm->nranks > 8) {
    return B200_ERR_INVALID_ARGUMENT;
  }
  auto* w = new (std::nothrow) b200_window;
  if (w == nullptr) return B200_ERR_INVALID_ARGUMENT;
  w->bytes = bytes;
  w->nranks = comm->nranks;
  w->rank = comm->rank;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  auto fail = [&](int rc) {
    for (int r = 0; r < w->nranks; ++r) {
      if (r != w->rank && w->peer[r] != nullptr) cudaIpcCloseMemHandle(w->peer[r]);
    }
    if (w->local) cudaFree(w->local);
    if (w->token) cudaFree(w->token);
    delete w;
    return rc;
  };
  cudaError_t e = cudaMalloc(&w->local, bytes);
  if (e != cudaSuccess) {
    w->local = nullptr;
    return fail(int(e));
  }
  w->peer[w->rank] = w->local;
  e = cudaMemsetAsync(w->local, 0, bytes, s);
  if (e != cudaSuccess) return fail(int(e));
  e = cudaMalloc(&w->token, sizeof(int));
  if (e != cudaSuccess) {
    w->token = nullptr;
    return fail(int(e));
  }
  if (w->nranks > 1) {
    cudaIpcMemHandle_t mine;
    e = cudaIpcGetMemHandle(&mine, w->local);
    if (e != cudaSuccess) return fail(int(e));
    const size_t hb = sizeof(cudaIpcMemHandle_t);
    void* dev = nullptr;
    e = cudaMalloc(&dev, hb * w->nranks);
    if (e != cudaSuccess) return fail(int(e));
    std::vector<cudaIpcMemHandle_t> all(w->nranks);
    e = cudaMemcpyAsync(static_cast<char*>(dev) + hb * w->rank, &mine, hb,
                        cudaMemcpyHostToDevice, s);
    int rc = e == cudaSuccess ? B200_OK : int(e);
    if (rc == B200_OK) {
      rc = b200::nccl_status(ncclAllGather(static_cast<char*>(dev) + hb * w->rank, dev, hb,
                                           ncclUint8, comm->nccl, s));
    }
    if (rc == B200_OK) {
      e = cudaMemcpyAsync(all.data(), dev, hb * w->nranks, cudaMemcpyDeviceToHost, s);
      if (e == cudaSuccess) e = cudaStreamSynchronize(s);
      rc = e == cudaSuccess ? B200_OK : int(e);
    }
    cudaFree(dev);
    if (rc != B200_OK) return fail(rc);
    for (int r = 0; r < w->nranks; ++r) {
      if (r == w->rank) continue;
      e = cudaIpcOpenMemHandle(&w->peer[r], all[r], cudaIpcMemLazyEnablePeerAccess);
      if (e != cudaSuccess) {
        w->peer[r] = nullptr;
        return fail(int(e));
      }
    }
  }
  *out = w;
  return B200_OK;
}

void* b200_window_ptr(b200_window_t w) { return w == nullptr ? nullptr : w->local; }

int b200_window_destroy(b200_window_t w) {
  if (w == nullptr) return B200_OK;
  cudaError_t first = cudaSuccess;
  for (int r = 0; r < w->nranks; ++r) {
    if (r != w->rank && w->peer[r] != nullptr) {
      const cudaError_t e = cudaIpcCloseMemHandle(w->peer[r]);
      if (first == cudaSuccess) first = e;
    }
  }
  cudaError_t e = cudaFree(w->local);
  if (first == cudaSuccess) first = e;
  e = cudaFree(w->token);
  if (first == cudaSuccess) first = e;
  delete w;
  return first == cudaSuccess ? B200_OK : int(first);
}

int b200_sharded_gemm_w8a16_p2p(b200_comm_t comm, b200_window_t out,
                                const int8_t* weight_shard, const uint16_t* scales_shard,
                                int group_size, const uint16_t* bias_shard,
                                const uint16_t* input, int tokens, int out_features,
                                int in_features, b200_stream_t stream) {
  if (group_size != 64) return B200_ERR_GROUP_SIZE;
  if (comm == nullptr || out == nullptr || tokens < 0 || out_features < 0 ||
      in_features <= 0 || out->nranks != comm->nranks || out->rank != comm->rank) {
    return B200_ERR_INVALID_ARGUMENT;
  }
  const int p = comm->nranks;
  if (out_features % p != 0) return B200_ERR_INVALID_ARGUMENT;
  const int ns = out_features / p;
  if (tokens == 0 || out_features == 0) return B200_OK;
  if (ns % 8 != 0 || out_features % 8 != 0) return B200_ERR_INVALID_ARGUMENT;
  if (weight_shard == nullptr || scales_shard == nullptr || input == nullptr) {
    return B200_ERR_INVALID_ARGUMENT;
  }
  if (size_t(tokens) * size_t(out_features) * 2 > out->bytes) return B200_ERR_WORKSPACE;
  if (!b200::gemm_tc_supported(true, weight_shard, input, out->local, tokens, ns,
                               in_features)) {
    return B200_ERR_INVALID_ARGUMENT;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // This rank's columns of the row-major [tokens, out_features] output.
  bf16* mine = static_cast<bf16*>(out->local) + size_t(comm->rank) * ns;
  b200::PeerOuts peers;
  for (int r = 0; r < p; ++r) {
    if (r == comm->rank) continue;
    peers.delta[peers.n++] =
        static_cast<char*>(out->peer[r]) - static_cast<char*>(out->local);
  }
  if (p > 1) {
    // Entry ordering point: no rank stores into a peer's window before every
    // rank has finished what its stream enqueued earlier, including reads of
    // the window's previous contents (the window is reused call after call).
    const int rc = b200::nccl_status(
        ncclAllReduce(out->token, out->token, 1, ncclInt32, ncclSum, comm->nccl, s));
    if (rc != B200_OK) return rc;
  }
  cudaError_t e = b200::launch_gemm_tc_peers(
      true, weight_shard, reinterpret_cast<const bf16*>(scales_shard),
      reinterpret_cast<const bf16*>(bias_shard), reinterpret_cast<const bf16*>(input), mine,
      tokens, ns, in_features, out_features, peers, s);
  if (e != cudaSuccess) return int(e);
  if (p > 1) {
    // Ordering point: a rank passes this all-reduce only after every rank's
    // GEMM (and so its stores into this rank's window) has completed.
    return b200::nccl_status(
        ncclAllReduce(out->token, out->token, 1, ncclInt32, ncclSum, comm->nccl, s));
  }
  return B200_OK;
}

size_t b200_sharded_gemm_workspace_bytes(int tokens, int out_features,
                                         int nranks) {
  if (tokens <= 0 || out_features <= 0 || nranks <= 0) return 0;
  return size_t(tokens) * size_t(out_features) * 2;
}

int b200_sharded_gemm_w8a16_allgather(
    b200_comm_t comm, const int8_t* weight_shard, const uint16_t* scales_shard,
    int group_size, const uint16_t* bias_shard, const uint16_t* input,
    uint16_t* output, void* workspace, int tokens, int out_features,
    int in_features, b200_stream_t stream) {
  if (group_size != 64) return B200_ERR_GROUP_SIZE;
  if (comm == nullptr || tokens < 0 || out_features < 0 || in_features <= 0) {
    return B200_ERR_INVALID_ARGUMENT;
  }
  const int p = comm->nranks;
  if (out_features % p != 0) return B200_ERR_INVALID_ARGUMENT;
  const int ns = out_features / p;
  if (tokens == 0 || out_features == 0) return B200_OK;
  if (ns % 8 != 0) return B200_ERR_INVALID_ARGUMENT;  // 16-byte slot rows
  if (weight_shard == nullptr || scales_shard == nullptr || input == nullptr ||
      output == nullptr || workspace == nullptr) {
    return B200_ERR_INVALID_ARGUMENT;
  }
  const size_t slot_elems = size_t(tokens) * ns;
  bf16* slots = static_cast<bf16*>(workspace);
  bf16* mine = slots + slot_elems * comm->rank;
  int rc = b200_gemm_w8a16(weight_shard, scales_shard, 64, bias_shard, input,
                           reinterpret_cast<uint16_t*>(mine), tokens, ns,
                           in_features, stream);
  if (rc != B200_OK) return rc;
  if (p > 1) {
    rc = b200::nccl_status(ncclAllGather(mine, slots, slot_elems * 2, ncclUint8,
                                         comm->nccl, stream));
    if (rc != B200_OK) return rc;
  }
  const int ns_vec = ns / 8;
  const size_t total = slot_elems * p / 8;
  int grid = int((total + 255) / 256);
  if (grid > 148 * 16) grid = 148 * 16;
  b200::gather_to_rows_kernel<<<grid, 256, 0, stream>>>(
      reinterpret_cast<const uint4*>(slots), reinterpret_cast<uint4*>(output),
      p, tokens, ns_vec);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? B200_OK : int(e);
}

size_t b200_sharded_lm_head_workspace_bytes(int vocab, int nranks) {
  if (vocab <= 0 || nranks <= 0) return 0;
  const size_t shard = size_t(vocab) / size_t(nranks);
  const size_t blocks = (shard + 7) / 8;
  // 8-byte key first (aligned), then the per-CTA partials.
  return 8 + blocks * (sizeof(float) + sizeof(int));
}

int b200_sharded_lm_head_bf16(b200_comm_t comm, const uint16_t* weight_shard,
                              const uint16_t* bias_shard,
                              const uint16_t* input, uint16_t* logits_shard,
                              void* workspace, int* argmax, int vocab,
                              int in_features, b200_stream_t stream) {
  if (comm == nullptr || vocab <= 0 || in_features < 0 || argmax == nullptr ||
      workspace == nullptr || logits_shard == nullptr) {
    return B200_ERR_INVALID_ARGUMENT;
  }
  const int p = comm->nranks;
  if (vocab % p != 0) return B200_ERR_INVALID_ARGUMENT;
  const int shard = vocab / p;
  if (in_features > 0 && (weight_shard == nullptr || input == nullptr)) {
    return B200_ERR_INVALID_ARGUMENT;
  }
  auto* key = static_cast<unsigned long long*>(workspace);
  float* block_value = reinterpret_cast<float*>(key + 1);
  const int blocks = (shard + 7) / 8;
  int* block_index = reinterpret_cast<int*>(block_value + blocks);
  int grid = 0;
  cudaError_t e = b200::launch_gemv(
      false, weight_shard, nullptr, reinterpret_cast<const bf16*>(bias_shard),
      reinterpret_cast<const bf16*>(input), reinterpret_cast<bf16*>(logits_shard),
      shard, in_features, block_value, block_index, stream, &grid);
  if (e != cudaSuccess) return int(e);
  if (grid > blocks) return B200_ERR_WORKSPACE;
  if (p > 1) {
    // Cross-GPU argmax through the key window (created on the first call,
    // collectively: every rank makes the same sequence of calls).
    if (comm->keys == nullptr) {
      const int rc = b200_window_create(comm, 2 * 2 * b200::kMaxRanks * sizeof(unsigned long long), stream,
                                        &comm->keys);
      if (rc != B200_OK) return rc;
    }
    b200::KeySlots slots;
    for (int q = 0; q < 8; ++q) {
      slots.slot[q] = static_cast<unsigned long long*>(q < p ? comm->keys->peer[q] : nullptr);
    }
    ++comm->seq;
    // Programmatic dependent launch: the exchange kernel is resident before
    // the GEMV finishes and waits for it in griddepcontrol.wait.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, b200::exchange_argmax_kernel, (const float*)block_value,
                           (const int*)block_index, grid, comm->rank * shard, slots, p,
                           comm->rank, comm->seq, argmax);
    return e == cudaSuccess ? B200_OK : int(e);
  }
  b200::local_argmax_key_kernel<<<1, 1024, 0, stream>>>(
      block_value, block_index, grid, comm->rank * shard, key);
  e = cudaGetLastError();
  if (e != cudaSuccess) return int(e);
  b200::decode_argmax_key_kernel<<<1, 1, 0, stream>>>(key, argmax);
  e = cudaGetLastError();
  return e == cudaSuccess ? B200_OK : int(e);
}

}  // extern "C"
