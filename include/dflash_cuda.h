/*
 * libdflashcuda — B200 (sm_100a) kernels for the speculative-decoding verify path of
 * random1st/dflash-swift (DFlashKit), behind a plain C ABI.
 *
 * Conventions for every entry point:
 *   - All tensor pointers are DEVICE pointers owned by the caller, unless a parameter
 *     says "host".  Nothing on the compute path allocates.
 *   - Calls are stream-ordered and asynchronous; none synchronises.
 *   - The return value is a status (DFLASH_OK == 0).  On failure
 *     dflash_last_error() (thread-local) describes it.  Nothing falls back to a CPU
 *     path: an unsupported shape or format returns DFLASH_ERR_UNSUPPORTED.
 *   - bf16 tensors are passed as dflash_bf16 (the raw 16-bit pattern of an IEEE
 *     bfloat16), so the header needs no CUDA include.
 *   - dflash_stream_t is binary-compatible with cudaStream_t; NULL is the legacy
 *     default stream.
 */
#ifndef DFLASH_CUDA_H
#define DFLASH_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef uint16_t dflash_bf16;
typedef struct CUstream_st* dflash_stream_t;

#define DFLASH_VERSION 1

enum dflash_status {
    DFLASH_OK = 0,
    DFLASH_ERR_INVALID_ARGUMENT = 1, /* null pointer, non-positive size, bad stride */
    DFLASH_ERR_UNSUPPORTED = 2,      /* bits / group size / row count the kernels do not cover */
    DFLASH_ERR_MISALIGNED = 3,       /* a pointer that must be 16-byte aligned is not */
    DFLASH_ERR_CUDA = 4,             /* a CUDA runtime or driver call failed */
    DFLASH_ERR_NCCL = 5,             /* an NCCL call failed */
    DFLASH_ERR_TIMEOUT = 6,          /* a bounded device-side wait ran out (see dflash_device_error) */
    DFLASH_ERR_WORKSPACE = 7         /* workspace missing or smaller than required */
};

/* Bits of the device error word (dflash_device_error). */
#define DFLASH_DEVERR_QMM_PIPELINE 0x1u   /* qmm TMA pipeline wait timed out */
#define DFLASH_DEVERR_QMM_REDUCE 0x2u     /* qmm split-K reduction inconsistency */
#define DFLASH_DEVERR_ALLREDUCE 0x4u      /* peer all-reduce flag wait timed out */
#define DFLASH_DEVERR_POSITION 0x8u       /* a device-resident cache position left the cache */
#define DFLASH_DEVERR_TEST_WAIT 0x80000000u /* raised only by dflash_test_bounded_wait */

int dflash_version(void);
const char* dflash_last_error(void);
const char* dflash_status_string(int status);

/* Reads the device error word of the current device into *bits (host pointer) and
 * clears it.  Synchronises the given stream.  A non-zero word means a kernel gave up
 * on a bounded wait and returned early; its outputs are not valid. */
int dflash_device_error(uint32_t* bits, dflash_stream_t stream);

/* Test hook for failure detection: launches one tiny kernel whose mbarrier wait can
 * never complete (nothing arrives), bounded at `limit_ns`; it records
 * DFLASH_DEVERR_TEST_WAIT in the device error word and returns.  Used only by the
 * test-suite to show a timed-out wait leaves the context usable. */
int dflash_test_bounded_wait(uint64_t limit_ns, dflash_stream_t stream);

/* ------------------------------------------------------------------------------
 * Small-M affine-quantized matmul.
 *
 * Replaces SmallMQuantizedMatmul.apply(x:weight:scales:biases:rows:outputFeatures:
 * inputFeatures:bits:) (Sources/DFlashKit/SmallMQuantizedMatmul.swift:210-224) and,
 * since it covers M = 1..16 and groups 32/64/128, the stock MLX call it stands in
 * for, quantizedMatmul(x, w, scales, biases, transpose: true, groupSize:, bits:)
 * (reached via QuantizedLinear, SmallMQuantizedMatmul.swift:265).
 *
 *   y[m, n] = sum_k x[m, k] * (q[n, k] * scales[n, k/g] + biases[n, k/g])
 *
 *   x       bf16 [M, K] row-major, 16-byte aligned
 *   w       uint32 [N, K*bits/32], MLX packing: low bits first within a word
 *           (SmallMQuantizedMatmul.swift:55-71), 16-byte aligned
 *   scales  bf16 [N, K/g], biases bf16 [N, K/g] (SmallMQuantizedMatmul.swift:127-129)
 *   y       bf16 [M, N] row-major (written, never read)
 *   M in 1..16, bits in {4, 8}, group_size in {32, 64, 128}, K % group_size == 0.
 *
 * The dequantised weight is exact (fp32 q*s+b), products accumulate in fp32, y is
 * rounded once to bf16.  `workspace` (16-byte aligned, sized by
 * dflash_qmm_workspace_bytes) receives x converted for the kernel; it needs no
 * initialisation, and each concurrently running stream needs its own.  The call is two
 * kernels chained by programmatic dependent launch: w, scales and biases are read
 * before the preceding kernel in the stream has finished, so they must not be written
 * by that kernel (x may be).
 * -------------------------------------------------------------------------------- */
size_t dflash_qmm_workspace_bytes(int M, int N, int K, int group_size, int bits);

int dflash_qmm(const dflash_bf16* x, const uint32_t* w, const dflash_bf16* scales,
               const dflash_bf16* biases, dflash_bf16* y, int M, int N, int K, int group_size,
               int bits, void* workspace, size_t workspace_bytes, dflash_stream_t stream);

/* dflash_qmm for callers that cannot allocate device memory (no counterpart in the
 * reference, whose MLX runtime always owns allocation): code running inside a CUDA
 * graph capture it does not control, plugin hosts whose allocator is off limits, or
 * latency-critical paths where a cudaMalloc could block or fail.  Same arguments and
 * results as dflash_qmm, without `workspace`: the scratch is a library-owned 8 MiB
 * device array that every GPU loading this library keeps until the process exits.
 *   - Shapes whose dflash_qmm_workspace_bytes exceeds 8 MiB are rejected with
 *     DFLASH_ERR_UNSUPPORTED (at M = 16 and group 32 that is K above about 209000;
 *     dflash_qmm with a larger workspace covers those).
 *   - The first call on a device resolves the array's device address; make that first
 *     call outside any stream capture.  A later call in a new context on that device
 *     (after cudaDeviceReset) resolves it again, so it too belongs outside a capture.
 *   - Every call on a device shares the array: calls that can overlap on the GPU
 *     (different streams without ordering between them) race and corrupt each other's
 *     results.  Keep such calls on one stream, or use dflash_qmm with one workspace per
 *     stream.
 *   - Calls allocate nothing (no cudaMalloc, cudaFree or library allocator). */
int dflash_qmm_noalloc(const dflash_bf16* x, const uint32_t* w, const dflash_bf16* scales,
                       const dflash_bf16* biases, dflash_bf16* y, int M, int N, int K, int group_size,
                       int bits, dflash_stream_t stream);

/* dflash_qmm with x and y in HOST memory (the call a host makes when its activations
 * live on the CPU side, e.g. a ctypes or Swift host holding MLX-style arrays): on
 * `stream` it copies x in, runs the matmul, and copies y out, so the host issues one
 * call instead of a copy, a matmul and a copy.  w, scales and biases are device memory as
 * for dflash_qmm.  The workspace (device, 16-byte aligned) also holds the device copies of
 * x and y: dflash_qmm_host_workspace_bytes gives its size (0 for an unsupported shape).
 * Pinned host buffers (cudaHostAlloc / cudaHostRegister) make the copies asynchronous;
 * y_host holds the result once the stream has run past the call (an event recorded
 * after it, or a stream synchronise).  Give each stream its own workspace. */
size_t dflash_qmm_host_workspace_bytes(int M, int N, int K, int group_size, int bits);
int dflash_qmm_host(const dflash_bf16* x_host, const uint32_t* w, const dflash_bf16* scales,
                    const dflash_bf16* biases, dflash_bf16* y_host, int M, int N, int K, int group_size,
                    int bits, void* workspace, size_t workspace_bytes, dflash_stream_t stream);

/* y bf16 [rows, N] += bias bf16 [N], rounded to bf16 per element: the optional bias of a
 * quantized linear layer, added after the matmul (SmallMQuantizedLinear.callAsFunction,
 * SmallMQuantizedMatmul.swift:287-290). */
int dflash_bias_add(dflash_bf16* y, const dflash_bf16* bias, int rows, int N, dflash_stream_t stream);

/* Static half of the reference's eligibility test (SmallMQuantizedMatmul.isEligible,
 * SmallMQuantizedMatmul.swift:193-201) for a layer of this library: 1 when
 * dflash_qmm covers (N, K, group_size, bits) for every M in 1..16, else 0.  Wider
 * than the reference's gate (which requires group 64, N >= 4096, K % 512 == 0). */
int dflash_qmm_supported(int N, int K, int group_size, int bits);

/* ------------------------------------------------------------------------------
 * Gated-delta recurrence: verify-time step with capture, and rollback replay.
 *
 * Per head the state S is fp32 [dv, dk] (dk contiguous).  One position t does
 *     S <- alpha_t * S;  u <- v_t - S k_t;  S <- S + beta_t * u k_t^T;  o_t <- S (q_scale * q_t)
 * Layouts for one layer: q, k [T, H, dk] bf16; v [T, H, dv] bf16; alpha, beta [T, H]
 * fp32; state [H, dv, dk] fp32; out [T, H, dv] bf16.
 * -------------------------------------------------------------------------------- */

/* The committed/verify forward of one gated-delta layer over T positions.  Reads
 * state_in (the pre-round snapshot, left untouched) and writes the state after the
 * T positions to state_out (ping-pong buffers; they must not overlap).  q, k, v,
 * alpha and beta are exactly what a later dflash_gdn_replay needs, so keeping them is
 * the capture (mtpGatedDeltaCaptureFlagKey, DFlashSpeculativeGenerator.swift:391-393).
 * out may be NULL when only the state is wanted. */
int dflash_gdn_step(const float* state_in, float* state_out, const dflash_bf16* q,
                    const dflash_bf16* k, const dflash_bf16* v, const float* alpha,
                    const float* beta, dflash_bf16* out, int T, int heads, int dk, int dv,
                    float q_scale, dflash_stream_t stream);

/* The verify forward of one gated-delta layer over the T rows of a speculative tree
 * round (the target forward run with mtpTreePlanKey, SpeculativeTreeTests.swift:108-140):
 * parents (device int32 [T], read in stream order) gives each row's parent row, -1 for
 * the anchor row 0 and an earlier row otherwise (a malformed entry makes its row a root).
 * Row t's output is that of a chain step over its root-to-t path from state_in, the
 * pre-round snapshot, which is left untouched; no state is written, since the state
 * after the round is the replay (dflash_gdn_replay) of the accepted path's rows.
 * Layouts as for dflash_gdn_step; 1 <= T <= 32. */
int dflash_gdn_step_tree(const float* state_in, const dflash_bf16* q, const dflash_bf16* k,
                         const dflash_bf16* v, const float* alpha, const float* beta,
                         const int32_t* parents, dflash_bf16* out, int T, int heads, int dk, int dv,
                         float q_scale, dflash_stream_t stream);

/* Layers whose q and k have fewer heads than v (k_heads key heads, each shared by
 * heads / k_heads consecutive value heads: value head h reads key head
 * h / (heads / k_heads)), as the target's Qwen3.5 configuration allows
 * (linear_num_key_heads < linear_num_value_heads,
 * Tests/DFlashKitTests/TinyHybridTarget.swift:27-30).  Same as the entries above with q
 * and k laid out [T, k_heads, dk] (replay: [layers, width, k_heads, dk]); v, alpha, beta,
 * out and the state keep `heads` value heads.  k_heads must divide heads; k_heads ==
 * heads is the ungrouped entry. */
int dflash_gdn_step_grouped(const float* state_in, float* state_out, const dflash_bf16* q,
                            const dflash_bf16* k, const dflash_bf16* v, const float* alpha,
                            const float* beta, dflash_bf16* out, int T, int heads, int k_heads, int dk,
                            int dv, float q_scale, dflash_stream_t stream);
int dflash_gdn_step_tree_grouped(const float* state_in, const dflash_bf16* q, const dflash_bf16* k,
                                 const dflash_bf16* v, const float* alpha, const float* beta,
                                 const int32_t* parents, dflash_bf16* out, int T, int heads, int k_heads,
                                 int dk, int dv, float q_scale, dflash_stream_t stream);
int dflash_gdn_replay_grouped(const float* snapshot, float* state_out, const dflash_bf16* k,
                              const dflash_bf16* v, const float* alpha, const float* beta,
                              const int32_t* rows, int keep, int width, int layers, int heads, int k_heads,
                              int dk, int dv, dflash_stream_t stream);

/* Rollback of a verify round for `layers` gated-delta layers at once
 * (rollbackGatedDeltaRound / rollbackGatedDeltaTree, called at
 * DFlashSpeculativeGenerator.swift:455-460).  From the pre-round snapshot, replays
 * the captured inputs of positions rows[0..keep-1] (host array; NULL means the chain
 * 0..keep-1) and writes the rebuilt state to state_out.
 *   snapshot, state_out: fp32 [layers, H, dv, dk]
 *   k: bf16 [layers, width, H, dk]; v: bf16 [layers, width, H, dv]
 *   alpha, beta: fp32 [layers, width, H]
 * 1 <= keep <= width <= 64; every rows[i] in [0, width). */
int dflash_gdn_replay(const float* snapshot, float* state_out, const dflash_bf16* k,
                      const dflash_bf16* v, const float* alpha, const float* beta,
                      const int32_t* rows, int keep, int width, int layers, int heads, int dk,
                      int dv, dflash_stream_t stream);

/* Conv-window rebuild for the same rollback (MambaCache slot 0 in
 * Tests/DFlashKitTests/GatedDeltaRollbackTests.swift:90-95): new window = last kc1
 * rows of [window || conv_in[rows[0..keep-1]]], for `layers` layers at once.
 *   window, window_out: bf16 [layers, kc1, channels]
 *   conv_in: bf16 [layers, width, channels] (the round's pre-conv inputs)
 * rows is a host array or NULL (chain).  window_out must not overlap window. */
int dflash_gdn_conv_rollback(const dflash_bf16* window, dflash_bf16* window_out,
                             const dflash_bf16* conv_in, const int32_t* rows, int keep, int width,
                             int layers, int kc1, int channels, dflash_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* DFLASH_CUDA_H */
