/*
 * libdflashcuda — glue kernels of the tensor-parallel verify stack (a hybrid
 * gated-delta / attention target around the quantized projections of dflash_cuda.h).
 * These have no single counterpart in the reference: there the same steps are MLX ops
 * inside the target model's layers (the verify forward of
 * Sources/DFlashKit/DFlashSpeculativeGenerator.swift:389-398).  Conventions as in
 * dflash_cuda.h: device pointers, row-major with one row per token, stream-ordered,
 * status return.
 */
#ifndef DFLASH_STACK_H
#define DFLASH_STACK_H

#include "dflash_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

/* resid (fp32 [M, H]) += delta (bf16 [M, H], NULL for none); out (bf16 [M, H]) =
 * resid * rsqrt(mean(resid^2) + eps) * weight (bf16 [H]). */
int dflash_stack_add_rmsnorm(float* resid, const dflash_bf16* delta, const dflash_bf16* weight, dflash_bf16* out,
                             int M, int H, float eps, dflash_stream_t stream);

/* gate_up bf16 [M, 2I] = [gate | up]; y bf16 [M, I] = silu(gate) * up. */
int dflash_stack_silu_mul(const dflash_bf16* gate_up, dflash_bf16* y, int M, int I, dflash_stream_t stream);

/* Causal depthwise convolution (width kc <= 8) over the M tokens of x (bf16, row stride ld,
 * channels [0, C)) continuing the pre-round `window` (bf16 [kc-1, C], read only), then
 * SiLU.  weight bf16 [C, kc] (last tap on the current token).  y receives `parts`
 * contiguous blocks [M, C / parts]. */
int dflash_stack_conv_silu(const dflash_bf16* x, int ld, const dflash_bf16* window, const dflash_bf16* weight,
                           dflash_bf16* y, int M, int C, int kc, int parts, dflash_stream_t stream);

/* Gated-delta gates: L2-normalise q and k (bf16 [M, heads * dk], in place); from ab (bf16,
 * row stride ld_ab, b at [0, heads), a at [heads, 2 heads)) write fp32 [M, heads]
 * alpha = exp(-exp(a_log) * softplus(a + dt_bias)) and beta = sigmoid(b). */
int dflash_stack_gdn_gates(dflash_bf16* q, dflash_bf16* k, const dflash_bf16* ab, int ld_ab, const float* a_log,
                           const float* dt_bias, float* alpha, float* beta, int M, int heads, int dk,
                           dflash_stream_t stream);

/* dflash_stack_conv_silu (parts = 3) followed by dflash_stack_gdn_gates on its q and k, in
 * one kernel with the same results: x rows hold the q|k|v channels at [0, 3 heads dk);
 * y receives the three [M, heads dk] blocks (q, k normalised); ab, a_log, dt_bias, alpha,
 * beta as for the gates.  dk in {32, 64, 128}, kc in 2..4. */
int dflash_stack_gdn_conv_gates(const dflash_bf16* x, int ld, const dflash_bf16* window, const dflash_bf16* weight,
                                dflash_bf16* y, const dflash_bf16* ab, int ld_ab, const float* a_log,
                                const float* dt_bias, float* alpha, float* beta, int M, int heads, int dk, int kc,
                                dflash_stream_t stream);

/* dflash_stack_gdn_conv_gates for layers whose q and k have k_heads heads and v has `heads`
 * (k_heads divides heads; see dflash_gdn_step_grouped): x rows hold
 * [q (k_heads dk) | k (k_heads dk) | v (heads dk)], weight and window cover those
 * (2 k_heads + heads) dk channels, y receives [q: M x k_heads dk | k: M x k_heads dk |
 * v: M x heads dk], and the gates (ab: b then a, one per value head) go to alpha, beta
 * fp32 [M, heads].  parents: NULL for a chain round, else a tree round's parent list
 * (M <= 32) as for dflash_stack_gdn_conv_gates_tree. */
int dflash_stack_gdn_conv_gates_grouped(const dflash_bf16* x, int ld, const dflash_bf16* window,
                                        const dflash_bf16* weight, dflash_bf16* y, const dflash_bf16* ab, int ld_ab,
                                        const float* a_log, const float* dt_bias, float* alpha, float* beta, int M,
                                        int heads, int k_heads, int dk, int kc, const int32_t* parents,
                                        dflash_stream_t stream);

/* out bf16 [M, heads * dv] = rmsnorm(o per head) * weight (bf16 [dv]) * silu(z); z has row
 * stride ld_z. */
int dflash_stack_gated_norm(const dflash_bf16* o, const dflash_bf16* z, int ld_z, const dflash_bf16* weight,
                            dflash_bf16* out, int M, int heads, int dv, float eps, dflash_stream_t stream);

/* Attention prep.  qkv row t (stride ld) = [q (hq*d) | gate (hq*d) | k (hkv*d) | v (hkv*d)].
 * q heads: RMSNorm (q_norm, bf16 [d]) then rotary embedding on the first rot dims, in
 * place.  k heads: RMSNorm (k_norm) + rotary into cache_k[j, pos0 + t]; v into
 * cache_v[j, pos0 + t].  Caches bf16 [hkv, max_len, d].  Rotary is rotate-half with
 * frequency theta^(-2i/rot).  d in {64, 128, 256}; rot a multiple of 64, <= d. */
int dflash_stack_attn_prep(dflash_bf16* qkv, int ld, const dflash_bf16* q_norm, const dflash_bf16* k_norm,
                           dflash_bf16* cache_k, dflash_bf16* cache_v, int M, int hq, int hkv, int d, int rot,
                           int pos0, int max_len, float eps, float theta, dflash_stream_t stream);

/* Decode attention of the block: token t attends to cache rows 0 .. pos0 + t of kv head
 * h / (hq / hkv).  out bf16 [M, hq * d] = softmax(q k^T * scale) v * sigmoid(gate), with q
 * and gate read from qkv as laid out above. */
int dflash_stack_attn_decode(const dflash_bf16* qkv, int ld, const dflash_bf16* cache_k, const dflash_bf16* cache_v,
                             dflash_bf16* out, int M, int hq, int hkv, int d, int pos0, int max_len, float scale,
                             dflash_stream_t stream);

/* dflash_stack_attn_prep / dflash_stack_attn_decode with both options at once: `parents`
 * (NULL: a chain round; else a tree round as for the _tree entries, M <= 32) and
 * `position` (NULL: pos0 as given; else a device int32 holding pos0, read in stream order,
 * so a CUDA graph of the round replays at whatever position the host last wrote there).
 * A device position outside 0 .. max_len - M makes the kernel write nothing and raise
 * DFLASH_DEVERR_POSITION in the device error word. */
int dflash_stack_attn_prep_ex(dflash_bf16* qkv, int ld, const dflash_bf16* q_norm, const dflash_bf16* k_norm,
                              dflash_bf16* cache_k, dflash_bf16* cache_v, int M, int hq, int hkv, int d, int rot,
                              int pos0, int max_len, float eps, float theta, const int32_t* parents,
                              const int32_t* position, dflash_stream_t stream);
int dflash_stack_attn_decode_ex(const dflash_bf16* qkv, int ld, const dflash_bf16* cache_k,
                                const dflash_bf16* cache_v, dflash_bf16* out, int M, int hq, int hkv, int d, int pos0,
                                int max_len, float scale, const int32_t* parents, const int32_t* position,
                                dflash_stream_t stream);

/* ------------------------------------------------------------------------------
 * Speculative tree rounds (the target forward run with mtpTreePlanKey,
 * Tests/DFlashKitTests/SpeculativeTreeTests.swift:108-140).  The M block rows carry a
 * parent list `parents` (device int32 [M], read in stream order, so a CUDA graph can be
 * replayed with a new tree): -1 for the anchor row 0, an earlier row otherwise (a
 * malformed entry makes its row a root).  Each row computes what a chain over its
 * root-to-row path computes: M <= 32.
 * -------------------------------------------------------------------------------- */

/* dflash_stack_gdn_conv_gates over a tree: tap i of row t reads its ancestor kc-1-i steps
 * up, and the window where that path runs past the anchor. */
int dflash_stack_gdn_conv_gates_tree(const dflash_bf16* x, int ld, const dflash_bf16* window,
                                     const dflash_bf16* weight, dflash_bf16* y, const dflash_bf16* ab, int ld_ab,
                                     const float* a_log, const float* dt_bias, float* alpha, float* beta, int M,
                                     int heads, int dk, int kc, const int32_t* parents, dflash_stream_t stream);

/* dflash_stack_attn_prep over a tree: rotary position pos0 + depth(t); k and v still go
 * to cache row pos0 + t. */
int dflash_stack_attn_prep_tree(dflash_bf16* qkv, int ld, const dflash_bf16* q_norm, const dflash_bf16* k_norm,
                                dflash_bf16* cache_k, dflash_bf16* cache_v, int M, int hq, int hkv, int d, int rot,
                                int pos0, int max_len, float eps, float theta, const int32_t* parents,
                                dflash_stream_t stream);

/* dflash_stack_attn_decode over a tree: token t attends to cache rows 0 .. pos0 - 1 and to
 * pos0 + a for each row a on its root-to-t path (the tree attention mask,
 * SpeculativeTreeTests.swift:50-66). */
int dflash_stack_attn_decode_tree(const dflash_bf16* qkv, int ld, const dflash_bf16* cache_k,
                                  const dflash_bf16* cache_v, dflash_bf16* out, int M, int hq, int hkv, int d,
                                  int pos0, int max_len, float scale, const int32_t* parents,
                                  dflash_stream_t stream);

/* The accepted path of a tree round on the device (DFlashDraftTree.acceptedPath,
 * Sources/DFlashKit/DFlashDraftTree.swift:122-141), so a captured round needs no host
 * round trip before its result is read: from the anchor, step into the first child (row
 * order) whose drafted token tokens[c] equals target_tokens[row] (the target's argmax at
 * the current row, as dflash_accept / dflash_accept_reduce write it), until none does.
 * Writes path[0 .. *path_len - 1] (anchor first; path needs `rows` entries), *path_len,
 * and *next_token = target_tokens[last row].  All device int32; 1 <= rows <= 32. */
int dflash_accept_tree(const int32_t* target_tokens, const int32_t* parents, const int32_t* tokens, int rows,
                       int32_t* path, int32_t* path_len, int32_t* next_token, dflash_stream_t stream);

/* After a tree round: moves cache rows pos0 + rows[i] to pos0 + i (i < keep) in cache_k
 * and cache_v, so the accepted path sits where a chain round would have put it (its
 * rotary positions pos0 + depth already match).  Caches bf16 [layers][hkv][max_len][d]
 * with layer_stride elements between layers (0 when layers = 1); rows is a host array
 * with 1 <= keep <= 32 and pos0 + rows[i] < max_len. */
int dflash_stack_kv_compact(dflash_bf16* cache_k, dflash_bf16* cache_v, int layers, long long layer_stride, int hkv,
                            int d, int pos0, int max_len, const int32_t* rows, int keep, dflash_stream_t stream);

/* ------------------------------------------------------------------------------
 * Tensor-parallel all-reduce over peer memory (one process per GPU of one node).
 * Each rank allocates one exchange buffer (dflash_tp_exchange_alloc, sized by
 * dflash_tp_exchange_bytes for the world size and the [M, H] reduced), shares it through
 * CUDA IPC (dflash_ipc_get_handle / dflash_ipc_open_handle, 64-byte handles exchanged by
 * the host), and then, for every all-reduce, in stream order:
 *   dflash_tp_push(part, bases, ...)            this rank's bf16 [M, H] partial into slot
 *                                               `rank` of every rank's buffer (NVLink stores
 *                                               of 8-byte words: 2 bf16 + the exchange epoch)
 *   dflash_stack_add_rmsnorm_reduce(..., set)   waits until every word carries the epoch,
 *                                               adds bf16(sum of the partials in rank order)
 *                                               to resid and normalises it
 * with `set` alternating 0, 1 from one all-reduce to the next (the same sequence on every
 * rank) and the same [M, H] for both calls of an exchange.  bases[r] is rank r's buffer
 * as mapped in this process (bases[rank] = own).  The wait is bounded (about a second):
 * on timeout DFLASH_DEVERR_ALLREDUCE is raised in the device error word and the output
 * is not meaningful.  Every rank's buffer must be allocated (it starts zeroed) before any
 * rank's first push (a host barrier).  The reference runs on one GPU and has no
 * counterpart; no TMA or multicast is involved.
 * ------------------------------------------------------------------------------ */
size_t dflash_tp_exchange_bytes(int world, int M, int H);
int dflash_tp_exchange_alloc(size_t bytes, void** ptr);
int dflash_tp_exchange_free(void* ptr);
int dflash_ipc_get_handle(const void* ptr, void* handle64);
int dflash_ipc_open_handle(const void* handle64, void** ptr);
int dflash_ipc_close_handle(void* ptr);
int dflash_tp_push(const dflash_bf16* part, void* const* bases, int rank, int world, int M, int H, int set,
                   dflash_stream_t stream);
int dflash_stack_add_rmsnorm_reduce(float* resid, void* exchange, int world, int set, const dflash_bf16* weight,
                                    dflash_bf16* out, int M, int H, float eps, dflash_stream_t stream);

/* ------------------------------------------------------------------------------
 * dflash_qmm with an input transform and/or an output that goes to the peer exchange,
 * so the SwiGLU and the all-reduce push need no kernel of their own.
 *   x_swiglu: x is bf16 [M, 2K] = [gate | up] (row stride 2K) and the matmul input is
 *             bf16(silu(gate) * up), the same bits dflash_stack_silu_mul would write.
 *   push:     y is not written (may be NULL); the bf16 [M, N] result goes to slot `rank`
 *             of exchange set `set` of every rank's buffer exactly as dflash_tp_push would
 *             write it, to be summed by dflash_stack_add_rmsnorm_reduce (H = N).
 *   argmax_keys (uint64 [M], device): y is not written; instead row m's largest bf16
 *             output and its lowest index among equal maxima end in argmax_keys[m]
 *             (high word: the value's order key, low word: ~index), the LM head's argmax
 *             without writing [M, V] logits (zeroed by the call itself).  Exclusive with push.
 * Other arguments, the workspace and the errors are dflash_qmm's.  No counterpart in the
 * reference for push and SwiGLU (its MLP activation and, on one GPU, no all-reduce); the
 * argmax is the first half of its accept test (DFlashSpeculativeGenerator.swift:564).
 * ------------------------------------------------------------------------------ */
typedef struct dflash_qmm_options {
    int x_swiglu;
    int push;
    int rank, world, set;
    void* const* bases; /* [world] exchange buffers as mapped in this process */
    void* argmax_keys;  /* uint64 [M] or NULL: see below */
    int argmax_index_base; /* added to the row index in the keys: a vocabulary shard's first row */
} dflash_qmm_options;

int dflash_qmm_ex(const dflash_bf16* x, const uint32_t* w, const dflash_bf16* scales, const dflash_bf16* biases,
                  dflash_bf16* y, int M, int N, int K, int group_size, int bits, void* workspace,
                  size_t workspace_bytes, const dflash_qmm_options* opts, dflash_stream_t stream);

/* Greedy accept of a verify round (acceptedPrefix, DFlashSpeculativeGenerator.swift:555-571):
 * from the LM head's argmax keys of drafts + 1 rows, target_tokens[i] = argmax of row i
 * (int32 [drafts + 1]) and *accepted = the number of leading i < drafts with
 * proposals[i] == target_tokens[i].  All device pointers; one tiny kernel. */
int dflash_accept(const unsigned long long* argmax_keys, const int32_t* proposals, int drafts,
                  int32_t* target_tokens, int32_t* accepted, dflash_stream_t stream);

/* The accept of a round whose LM head is sharded by vocabulary over the ranks: every rank
 * computed the argmax keys of its rows (dflash_qmm_ex with argmax_keys and its shard's
 * first row as argmax_index_base) and pushed them, as bf16 [drafts + 1, 4] (8 bytes per
 * key), into an exchange buffer of its own for [drafts + 1, 4] (dflash_tp_push, H = 4).
 * This waits (bounded) for every rank's keys, keeps the largest per row (the global
 * argmax, lowest index among equal maxima) and computes target_tokens and *accepted as
 * dflash_accept does. */
int dflash_accept_reduce(void* exchange, int world, int set, const int32_t* proposals, int drafts,
                         int32_t* target_tokens, int32_t* accepted, dflash_stream_t stream);

/* ------------------------------------------------------------------------------
 * The verify stack as one object, for hosts that drive a verify round through this
 * library alone (the reference's generator runs its verify forward, LM head and accept
 * in-process: Sources/DFlashKit/DFlashSpeculativeGenerator.swift:389-398 and :555-571,
 * and its rollback with rollbackGatedDeltaRound, :455-460).  It sequences the entry
 * points above: per layer RMSNorm, the token mixer (gated delta: in-projection, conv +
 * gates, recurrence step, gated norm, out-projection; attention: qkv, prep, decode,
 * o-projection), RMSNorm, MLP (gate/up, then down with the SwiGLU folded into its input);
 * the row-sharded projections' partials are summed over the ranks through the peer
 * exchange (world > 1).  Chain rounds only (rows 0 .. keep-1 are accepted).
 *
 * Weights and state are this rank's shard in the caller's device memory, referenced, never
 * copied: the caller keeps them alive until dflash_stack_destroy.  dflash_stack_create
 * allocates the activations, the capture and the qmm workspace once (cudaMalloc); the
 * round entry points allocate nothing, are stream-ordered and may be captured in a CUDA
 * graph.  Exchange set-up (world > 1): each rank allocates two buffers with
 * dflash_tp_exchange_alloc, one for [block, hidden] and one for [block, 4] (the LM head's
 * argmax keys), shares them with dflash_ipc_get_handle / dflash_ipc_open_handle over the
 * host's own channel, and passes both arrays of mapped bases (entry `rank` its own
 * buffer); every rank's buffers must exist before any rank's first round.
 * ------------------------------------------------------------------------------ */
typedef struct dflash_qweight { /* one quantized projection: MLX affine layout, device memory */
    const uint32_t* w;          /* [N, K * bits / 32] */
    const dflash_bf16* scales;  /* [N, K / group] */
    const dflash_bf16* biases;  /* [N, K / group] */
    int N, K;
} dflash_qweight;

typedef struct dflash_stack_layer { /* one layer of this rank's shard (unused members NULL) */
    int attention;                    /* 0: gated delta, 1: attention */
    const dflash_bf16* ln;            /* [hidden] input RMSNorm weight */
    const dflash_bf16* post_ln;       /* [hidden] post-mixer RMSNorm weight */
    /* gated delta (heads h, key heads hk, dims dk = dv, conv kernel kc of the descriptor) */
    dflash_qweight in_proj;           /* rows [q (hk dk) | k (hk dk) | v (h dv) | z (h dv) | b (h) | a (h)], K = hidden */
    dflash_qweight out_proj;          /* [hidden, h dv] */
    const dflash_bf16* conv;          /* [(2 hk + h) dk, kc] */
    const float* a_log;               /* [h] */
    const float* dt_bias;             /* [h] */
    const dflash_bf16* gdn_norm;      /* [dv] */
    float* snapshot;                  /* [h, dv, dk] pre-round state, read by rounds, rewritten by commit */
    dflash_bf16* window;              /* [kc - 1, (2 hk + h) dk] conv window, rewritten by commit */
    /* attention (hq q heads, hkv kv heads, head_dim d of the descriptor) */
    dflash_qweight qkv;               /* rows [q (hq d) | gate (hq d) | k (hkv d) | v (hkv d)], K = hidden */
    dflash_qweight o_proj;            /* [hidden, hq d] */
    const dflash_bf16* q_norm;        /* [d] */
    const dflash_bf16* k_norm;        /* [d] */
    dflash_bf16* cache_k;             /* [hkv, max_len, d] */
    dflash_bf16* cache_v;             /* [hkv, max_len, d] */
    /* MLP (this rank's I units) */
    dflash_qweight gate_up;           /* rows [gate (I) | up (I)], K = hidden */
    dflash_qweight down;              /* [hidden, I] */
} dflash_stack_layer;

typedef struct dflash_stack_desc {
    int layers, hidden, block;        /* block: rows M verified per round (1..16) */
    int gdn_heads, gdn_key_heads, gdn_dk, gdn_dv, conv_kernel;  /* this rank's gated-delta heads */
    int attn_heads, kv_heads, head_dim, rotary_dim, max_len;    /* this rank's attention heads; cache rows */
    float rope_theta, eps;
    int group, bits;                  /* quantization of every projection */
    int rank, world;
    int vocab0;                       /* first vocabulary row of this rank's LM-head shard */
    const dflash_stack_layer* layer;  /* [layers], copied at creation */
    const dflash_bf16* final_norm;    /* [hidden] */
    dflash_qweight lm_head;           /* this rank's vocabulary shard, K = hidden */
    void* const* exchange;            /* [world] mapped [block, hidden] exchange buffers (world > 1) */
    void* const* key_exchange;        /* [world] mapped [block, 4] exchange buffers (world > 1) */
} dflash_stack_desc;

typedef struct dflash_stack dflash_stack;

/* Checks the shard's shapes and allocates the round buffers; context: tokens already in the
 * attention caches (the block's rows go to context .. context + block - 1). */
int dflash_stack_create(const dflash_stack_desc* desc, int context, dflash_stack** out);
/* The verify forward of one block: hidden bf16 [block, hidden] -> out bf16 [block, hidden]
 * (NULL: the stack's own buffer, dflash_stack_output), identical on every rank. */
int dflash_stack_forward(dflash_stack* s, const dflash_bf16* hidden, dflash_bf16* out, dflash_stream_t stream);
/* A whole verify round: the forward, the LM head reduced to argmax keys, the accept
 * (dflash_accept / dflash_accept_reduce): target_tokens int32 [block], *accepted; all device. */
int dflash_stack_verify(dflash_stack* s, const dflash_bf16* hidden, const int32_t* proposals, int32_t* target_tokens,
                        int32_t* accepted, dflash_stream_t stream);
/* After a round: rows (host int32 [keep], NULL for 0 .. keep-1; only a chain's rows are
 * accepted) become the committed state: every gated-delta snapshot is replayed over them
 * and its conv window rebuilt.  The attention caches already hold them. */
int dflash_stack_commit(dflash_stack* s, const int32_t* rows, int keep, dflash_stream_t stream);
/* The caches hold n more committed tokens (host-side position, at most max_len; a round
 * needs room for its block and fails with DFLASH_ERR_INVALID_ARGUMENT otherwise). */
int dflash_stack_advance(dflash_stack* s, int n);
int dflash_stack_context(const dflash_stack* s);
const dflash_bf16* dflash_stack_output(const dflash_stack* s);
void dflash_stack_destroy(dflash_stack* s);

#ifdef __cplusplus
}
#endif

#endif /* DFLASH_STACK_H */
