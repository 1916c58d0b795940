/*
 * b200_linear.h - C ABI of the B200 (sm_100a) Linear-layer kernels.
 *
 * Drop-in boundary for the reference engine's CUDA Linear interface
 * (reference include/infer/cuda_ops.hpp:24-55,102-103; implemented there in
 * src/cuda/kernels.cu:1540-1704).  Every entry point takes raw device
 * pointers, sizes and a CUDA stream; nothing here synchronises the stream
 * or keeps state between calls, except the device-side error word read by
 * b200_device_status, the fixed scratch array of b200_lm_head_bf16_noalloc,
 * the summation-order switch, and the BF16 weight buffer of the two-pass
 * W8A16 prefill (allocated only by an explicit b200_gemm_reserve_scratch; no
 * Linear call allocates device memory).  All work is enqueued
 * asynchronously on `stream`, exactly like the reference functions.
 *
 * Layouts (reference conventions, src/qwen2.cpp:231-330):
 *   weight  [out_features, in_features] row-major (BF16 bits, or int8)
 *   scales  [out_features, ceil(in_features / 64)] BF16 bits (W8A16)
 *   input   [tokens, in_features] row-major BF16 bits
 *   output  [tokens, out_features] row-major BF16 bits
 *   bias    [out_features] BF16 bits, or NULL
 * BF16 values are passed as uint16_t bit patterns.  Accumulation is FP32 and
 * every output is rounded to BF16 round-to-nearest-even.
 *
 * Return value: B200_OK (0); a negative B200_ERR_* code for an argument the
 * kernels do not accept (the reference throws infer::Error in those cases);
 * or a positive cudaError_t value from the launch.
 */
#ifndef B200_LINEAR_H_
#define B200_LINEAR_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same type as cudaStream_t (struct CUstream_st*), spelled without the CUDA
 * headers so that C/FFI callers need none.  NULL = the legacy default stream. */
typedef struct CUstream_st* b200_stream_t;

#define B200_OK 0
#define B200_ERR_INVALID_ARGUMENT (-1) /* NULL pointer, negative size */
#define B200_ERR_GROUP_SIZE (-2)       /* W8A16 group_size other than 64 */
#define B200_ERR_WORKSPACE (-3)        /* workspace missing or too small */
#define B200_ERR_TOO_LARGE (-4)        /* size beyond a stated limit */
#define B200_ERR_NCCL (-5)             /* NCCL call failed (sharded ops) */

/* Device-side error codes recorded by kernels whose bounded waits expired. */
#define B200_DEVICE_OK 0
#define B200_DEVICE_TIMEOUT_PIPELINE 1 /* GEMM smem pipeline wait expired */
#define B200_DEVICE_TIMEOUT_ACCUM 2    /* GEMM TMEM accumulator wait expired */
#define B200_DEVICE_TIMEOUT_GRID 3     /* persistent decode: wait for another CTA expired */

/* Library version (major*10000 + minor*100 + patch). */
int b200_version(void);

/* Human-readable text for a status returned by any b200_* function. */
const char* b200_status_string(int status);

/* Reads (and if clear != 0, resets) the device-side error word of the
 * current device.  Returns a B200_DEVICE_* code, or a negative B200_ERR_* /
 * the negated cudaError_t if the read itself failed.  Synchronises the
 * current device. */
int b200_device_status(int clear);

/* Summation order of the decode GEMVs and the fused LM heads.
 *   B200_ORDER_FAST (default): the fastest order per shape (FP32 throughout;
 *     outputs within one BF16 ulp of the reference, almost always equal).
 *   B200_ORDER_REFERENCE: every FP32 operation in the reference kernels'
 *     order, flushing denormals as the reference build does (--use_fast_math):
 *     one warp per row (four per row when a GEMV has in_features > 1024),
 *     16-element INT8 / 8-element BF16 chunks strided over the lanes, each
 *     chunk a fresh FMA chain, lane sums in chunk order, the __shfl_down tree,
 *     split-row partials in warp order (reference src/cuda/kernels.cu:359-384,
 *     438-490, 492-568, 953-1041).  Bit-identical outputs to the reference
 *     kernels on their fast paths (16-byte aligned weight and input,
 *     in_features % 8 == 0 for BF16, % 64 == 0 for W8A16) when out_features
 *     % 8 == 0; other shapes keep the fast order.  The prefill GEMMs need no
 *     mode: their tensor-core K order already gives the reference's results.
 * Process-wide; the initial value comes from the environment variable
 * B200_SUMMATION_ORDER ("reference" or "fast").  Affects launches made
 * after the call.  No reference counterpart (a numerics switch of this
 * library). */
#define B200_ORDER_FAST 0
#define B200_ORDER_REFERENCE 1
int b200_set_summation_order(int order);
int b200_summation_order(void);

/* Decode GEMV, BF16 weights: output[n] = bf16(sum_k W[n,k] x[k] + b[n]).
 * Replaces infer::cuda::gemv_bf16 (reference include/infer/cuda_ops.hpp:24-26,
 * src/cuda/kernels.cu:1540-1564).  Any out_features/in_features >= 0 and any
 * 2-byte alignment; the vectorised path needs in_features % 8 == 0 and
 * 16-byte aligned weight/input. */
int b200_gemv_bf16(const uint16_t* weight, const uint16_t* bias,
                   const uint16_t* input, uint16_t* output, int out_features,
                   int in_features, b200_stream_t stream);

/* Decode GEMV, W8A16 (group-64 INT8 weights, BF16 scales):
 * output[n] = bf16(sum_k float(q[n,k]) * s[n,k/64] * x[k] + b[n]).
 * Replaces infer::cuda::gemv_w8a16 (reference include/infer/cuda_ops.hpp:45-48,
 * src/cuda/kernels.cu:1627-1655).  group_size must be 64
 * (B200_ERR_GROUP_SIZE otherwise, checked before any pointer, as the
 * reference does at src/cuda/kernels.cu:1631). */
int b200_gemv_w8a16(const int8_t* weight, const uint16_t* scales,
                    int group_size, const uint16_t* bias,
                    const uint16_t* input, uint16_t* output, int out_features,
                    int in_features, b200_stream_t stream);

/* Prefill GEMM, BF16 weights: Y[m,n] = bf16(sum_k X[m,k] W[n,k] + b[n]).
 * Replaces infer::cuda::gemm_bf16 (reference include/infer/cuda_ops.hpp:32-35,
 * src/cuda/kernels.cu:1600-1625).  Tensor-core (tcgen05) path when
 * in_features % 8 == 0 and weight/input/output are 16-byte aligned;
 * otherwise a CUDA-core path with the same results within tolerance. */
int b200_gemm_bf16(const uint16_t* weight, const uint16_t* bias,
                   const uint16_t* input, uint16_t* output, int tokens,
                   int out_features, int in_features, b200_stream_t stream);

/* Prefill GEMM, W8A16: Y[m,n] = bf16(sum_k X[m,k] bf16(q[n,k] s[n,k/64]) + b[n])
 * (the dequantised weight is rounded to BF16 before the multiply, as the
 * reference's tensor-core GEMM does, src/cuda/kernels.cu:1075-1094).
 * Replaces infer::cuda::gemm_w8a16 (reference include/infer/cuda_ops.hpp:49-53,
 * src/cuda/kernels.cu:1657-1684).  group_size must be 64. */
int b200_gemm_w8a16(const int8_t* weight, const uint16_t* scales,
                    int group_size, const uint16_t* bias,
                    const uint16_t* input, uint16_t* output, int tokens,
                    int out_features, int in_features, b200_stream_t stream);

/* Allocates now, on the current device, the BF16 weight buffer (at most
 * 256 MiB, or `bytes` if smaller and non-zero) that b200_gemm_w8a16 may use
 * for large prefills (>= 1024 tokens and >= 2^25 outputs, where it measured
 * faster): the INT8 weights are dequantised once to bf16(q*s) and the tensor-core
 * BF16 GEMM runs on them (same results as the one-pass kernels).  A GEMM call
 * never allocates: without this reservation the one-pass kernels run (for
 * >= 1024 tokens the one that keeps the dequantised weights in tensor
 * memory).  Call it at start-up, outside stream capture.  The buffer is one
 * per device and shared: two such GEMMs running at the same time on
 * different streams would race on it, so keep large W8A16 GEMMs of a device
 * in stream order (the reference engine uses one stream).  No reference
 * counterpart (the reference allocates its prefill workspace at start-up,
 * src/qwen2.cpp:80-200). */
int b200_gemm_reserve_scratch(size_t bytes);

/* Weight pre-packing at upload (W8A16).  The reference uploads the INT8
 * weights as they are, row-major [N, K] (src/qwen2.cpp:56-78), and its notes
 * name packing at upload as the place for kernel-specific layouts
 * (docs/architecture.md:36).  b200_pack_w8a16 re-tiles them once into
 * [2 ceil(N/256)][ceil(K/128)] blocks of 16 KB.  Each block is 128 rows x
 * 128 K values in the 128-byte-swizzled layout the prefill kernels hold in
 * shared memory.  Blocks are zero-filled outside the matrix.
 * b200_gemm_w8a16_packed then fetches each block with one contiguous bulk
 * copy instead of a box of rows strided by K.  Scales stay in the reference
 * layout.  Results are bit-identical to b200_gemm_w8a16.
 * Requirements: in_features % 16 == 0; weight, packed and input 16-byte
 * aligned.  The packed buffer (b200_w8a16_packed_bytes) is the caller's;
 * packing runs asynchronously on `stream`. */
size_t b200_w8a16_packed_bytes(int out_features, int in_features);
int b200_pack_w8a16(const int8_t* weight, int out_features, int in_features, void* packed,
                    b200_stream_t stream);
int b200_gemm_w8a16_packed(const void* packed, const uint16_t* scales, int group_size,
                           const uint16_t* bias, const uint16_t* input, uint16_t* output,
                           int tokens, int out_features, int in_features,
                           b200_stream_t stream);

/* Bytes of workspace b200_lm_head_* need, split as the reference splits it:
 * ceil(vocab/8) floats followed by ceil(vocab/8) ints
 * (reference src/qwen2.cpp:193-198).  The kernels use at most that much. */
size_t b200_lm_head_workspace_bytes(int vocab, int in_features);

/* Fused LM head: writes all BF16 logits[v] = bf16(sum_k W[v,k] x[k] + b[v])
 * and *argmax = the index of the largest BF16-rounded logit, lowest index on
 * ties.  block_max_value / block_max_index are caller workspace of
 * ceil(vocab/8) entries each.  Replaces infer::cuda::lm_head_bf16 (reference
 * include/infer/cuda_ops.hpp:40-43, src/cuda/kernels.cu:1566-1579). */
int b200_lm_head_bf16(const uint16_t* weight, const uint16_t* bias,
                      const uint16_t* input, uint16_t* logits,
                      float* block_max_value, int* block_max_index,
                      int* argmax, int vocab, int in_features,
                      b200_stream_t stream);

/* W8A16 form of the fused LM head (GEMV dequant arithmetic), for the
 * synthetic 896->151936 INT8 shape.  The reference has no INT8 LM head; its
 * equivalent is gemv_w8a16 followed by argmax_bf16
 * (src/cuda/kernels.cu:1627-1655, 326-356). */
int b200_lm_head_w8a16(const int8_t* weight, const uint16_t* scales,
                       int group_size, const uint16_t* bias,
                       const uint16_t* input, uint16_t* logits,
                       float* block_max_value, int* block_max_index,
                       int* argmax, int vocab, int in_features,
                       b200_stream_t stream);

/* Argmax over n BF16 values, lowest index on ties; 0 when n <= 0.
 * Replaces infer::cuda::argmax_bf16 (reference include/infer/cuda_ops.hpp:102-103,
 * src/cuda/kernels.cu:326-356, 1534-1538). */
int b200_argmax_bf16(const uint16_t* values, int n, int* output,
                     b200_stream_t stream);

/* ------------------------------------------------------------------------
 * Column-sharded Linear across the GPUs of one node (one process per GPU,
 * NCCL over NVLink).  The reference is single-GPU; these are the sharded
 * forms of gemm_w8a16 and lm_head_bf16 (src/cuda/kernels.cu:1566-1579,
 * 1657-1684) for the large synthetic shapes.  A b200_comm_t wraps an NCCL
 * communicator whose rank r drives the current CUDA device of its process.
 * ------------------------------------------------------------------------ */
typedef struct b200_comm* b200_comm_t;

/* Size of an NCCL unique id (bytes) and a fresh id, made on one rank and
 * shared with the others out of band (e.g. torch.distributed). */
int b200_nccl_unique_id_bytes(void);
int b200_nccl_get_unique_id(void* out);

/* Creates a communicator of nranks (ncclCommInitRank) on the current device. */
int b200_comm_init(b200_comm_t* comm, const void* unique_id, int nranks,
                   int rank);
/* Wraps an existing ncclComm_t (not owned: b200_comm_destroy leaves it). */
int b200_comm_wrap(b200_comm_t* comm, void* nccl_comm, int nranks, int rank);
int b200_comm_destroy(b200_comm_t comm);

/* A symmetric window: `bytes` of device memory on every rank, each rank's
 * buffer mapped into every other rank's process (CUDA IPC over NVLink).
 * Collective over the communicator (every rank calls it with the same
 * bytes); the IPC handles are exchanged with an NCCL all-gather on `stream`,
 * which the call synchronises. */
typedef struct b200_window* b200_window_t;
int b200_window_create(b200_comm_t comm, size_t bytes, b200_stream_t stream,
                       b200_window_t* window);
/* This rank's buffer of the window (device pointer), or NULL. */
void* b200_window_ptr(b200_window_t window);
/* Unmaps the peers' buffers and frees this rank's buffer. */
int b200_window_destroy(b200_window_t window);

/* The fused form of b200_sharded_gemm_w8a16_allgather: the local
 * tensor-core GEMM stores each output tile straight into the window of
 * every rank (16-byte stores over NVLink from its epilogue, so the exchange
 * overlaps the math tile by tile).  Two 4-byte NCCL all-reduces on `stream`
 * order it: one before the GEMM (no rank writes into a window that another
 * rank's stream may still be reading from the previous call, so one window
 * can serve call after call) and one after it (every rank's stores land
 * before what follows on any rank's stream).  On
 * completion the window holds the full row-major Y[tokens, out_features] on
 * every rank; the window must hold at least tokens x out_features BF16.
 * No gather workspace and no layout copy.  Same arguments and limits
 * otherwise. */
int b200_sharded_gemm_w8a16_p2p(b200_comm_t comm, b200_window_t output,
                                const int8_t* weight_shard,
                                const uint16_t* scales_shard, int group_size,
                                const uint16_t* bias_shard,
                                const uint16_t* input, int tokens,
                                int out_features, int in_features,
                                b200_stream_t stream);

/* Gather workspace of b200_sharded_gemm_w8a16_allgather: tokens x
 * out_features BF16 (the [P][tokens][out_features/P] slots). */
size_t b200_sharded_gemm_workspace_bytes(int tokens, int out_features,
                                         int nranks);

/* Y[tokens, out_features] = X . W^T + b with W split by rows across ranks:
 * this rank passes its rows [rank*N/P, (rank+1)*N/P) of W, of the scales and
 * of the bias; every rank receives the full row-major Y.  out_features must
 * be a multiple of 8 * nranks.  Enqueues the local tensor-core GEMM, an
 * NCCL all-gather and a layout copy on `stream`. */
int b200_sharded_gemm_w8a16_allgather(
    b200_comm_t comm, const int8_t* weight_shard, const uint16_t* scales_shard,
    int group_size, const uint16_t* bias_shard, const uint16_t* input,
    uint16_t* output, void* workspace, int tokens, int out_features,
    int in_features, b200_stream_t stream);

/* Workspace of b200_sharded_lm_head_bf16 (bytes, 8-byte aligned). */
size_t b200_sharded_lm_head_workspace_bytes(int vocab, int nranks);

/* Vocabulary-sharded fused LM head: this rank holds vocabulary rows
 * [rank*V/P, (rank+1)*V/P) and writes their BF16 logits to logits_shard;
 * every rank receives in *argmax the global index of the largest BF16 logit,
 * lowest index on ties.  With P > 1 the ranks exchange packed 64-bit keys
 * through a small window of NVLink-mapped slots that the communicator
 * creates on the first call (collective and synchronising: not inside a
 * stream capture the first time); one kernel per rank publishes its key and
 * reduces all P (bounded wait; an expired wait is reported by
 * b200_device_status).  vocab must be a multiple of nranks. */
int b200_sharded_lm_head_bf16(b200_comm_t comm, const uint16_t* weight_shard,
                              const uint16_t* bias_shard,
                              const uint16_t* input, uint16_t* logits_shard,
                              void* workspace, int* argmax, int vocab,
                              int in_features, b200_stream_t stream);

/* Fused LM head that allocates nothing and needs no workspace.
 * No counterpart in the reference (its lm_head_bf16 takes a caller-owned
 * workspace).  For callers that cannot allocate device memory -- a plugin
 * host that passes only inputs and outputs, or code already recording a CUDA
 * graph, where cudaMalloc is not allowed -- the per-CTA argmax partials live
 * in a fixed 256 KiB array in device memory owned by the library (one copy
 * per GPU that loads the library, held until the process exits).  Same
 * results as b200_lm_head_bf16.
 *   - vocab must be <= b200_lm_head_noalloc_max_vocab() (262144);
 *     larger returns B200_ERR_TOO_LARGE.
 *   - The first call on a device looks up that device's copy of the array
 *     (cudaGetSymbolAddress, with the device current); make that first call
 *     before any stream capture.
 *   - Every call on a device shares the one array: calls that may overlap on
 *     the GPU (different streams without ordering) race on it; order them.
 *   - No cudaMalloc, cudaFree or allocating library routine is called. */
size_t b200_lm_head_noalloc_max_vocab(void);
int b200_lm_head_bf16_noalloc(const uint16_t* weight, const uint16_t* bias,
                              const uint16_t* input, uint16_t* logits,
                              int* argmax, int vocab, int in_features,
                              b200_stream_t stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* B200_LINEAR_H_ */
