// The tensor-parallel verify stack as one C-ABI object (dflash_stack_*, include/dflash_stack.h):
// a host that is not Python (the reference's Swift generator, a C++ server) runs a verify
// round through libdflashcuda alone.  It sequences the library's own entry points exactly
// as the reference's verify forward sequences its layers
// (Sources/DFlashKit/DFlashSpeculativeGenerator.swift:389-398: the target run over the
// M-row block, the LM head and the greedy accept, :555-571) and, after the round, the
// rollback of every gated-delta layer to the accepted rows (rollbackGatedDeltaRound,
// :455-460).  Weights and state are the caller's device buffers (this rank's shard); the
// object owns only the activations, the capture and the qmm workspace, allocated once at
// creation, so a round allocates nothing.  Tensor-parallel ranks exchange partial sums over
// peer memory: the caller allocates the exchange buffers with dflash_tp_exchange_alloc,
// swaps their IPC handles through its own channel and passes the mapped bases.
#include "common.cuh"
#include "dflash_stack.h"

#include <cmath>
#include <new>
#include <vector>

struct dflash_stack {
    dflash_stack_desc d;
    std::vector<dflash_stack_layer> layer;
    int context;
    // activations
    float* resid = nullptr;        // fp32 [M, H]
    dflash_bf16* normed = nullptr;  // [M, H]
    dflash_bf16* delta = nullptr;   // [M, H]: a row-sharded projection's output at world 1
    dflash_bf16* out = nullptr;     // [M, H]: the final norm's output
    unsigned long long* keys = nullptr;  // [M]
    dflash_bf16* gdn_o = nullptr;       // [M, h, dv]
    dflash_bf16* gdn_normed = nullptr;  // [M, h dv]
    dflash_bf16* qkv = nullptr;         // [M, (2 hq + 2 hkv) d]
    dflash_bf16* attn_out = nullptr;    // [M, hq d]
    dflash_bf16* gate_up = nullptr;     // [M, 2 I]
    dflash_bf16* conv_in = nullptr;     // [M, C]: commit's contiguous copy of a layer's conv inputs
    dflash_bf16* window_tmp = nullptr;  // [kc - 1, C]
    // capture, per gated-delta layer
    std::vector<dflash_bf16*> proj;  // [M, n_in]: the in-projection (its first C channels are the conv inputs)
    std::vector<dflash_bf16*> cqkv;  // [q: M x hk dk | k: M x hk dk | v: M x h dk]
    std::vector<float*> alpha, beta;  // [M, h]
    std::vector<float*> state_out;    // [h, dv, dk]
    void* ws = nullptr;
    size_t ws_bytes = 0;
    std::vector<void*> allocations;
    int set = 0;  // the exchange set of the next all-reduce (alternates on every rank alike)
};

namespace dflash {
namespace stackdrv {

int n_in(const dflash_stack_desc& d) {
    return 2 * d.gdn_key_heads * d.gdn_dk + 2 * d.gdn_heads * d.gdn_dv + 2 * d.gdn_heads;
}
int conv_channels(const dflash_stack_desc& d) { return (2 * d.gdn_key_heads + d.gdn_heads) * d.gdn_dk; }

template <class T>
int alloc(dflash_stack* s, T** p, size_t count) {
    void* v = nullptr;
    DFLASH_CUDA_TRY(cudaMalloc(&v, count * sizeof(T) > 0 ? count * sizeof(T) : 16));
    s->allocations.push_back(v);
    *p = static_cast<T*>(v);
    return DFLASH_OK;
}

bool quant_ok(const dflash_qweight& q, int N, int K) {
    return q.w && q.scales && q.biases && q.N == N && q.K == K;
}

// What the next norm adds: a local partial, or the peer exchange set it was pushed into.
struct Pending {
    const dflash_bf16* delta;
    int exchange_set;  // -1: `delta`
};

int norm(dflash_stack* s, const Pending& pd, const dflash_bf16* weight, dflash_bf16* out, cudaStream_t st) {
    const dflash_stack_desc& d = s->d;
    if (pd.exchange_set >= 0)
        return dflash_stack_add_rmsnorm_reduce(s->resid, d.exchange[d.rank], d.world, pd.exchange_set, weight, out,
                                               d.block, d.hidden, d.eps, st);
    return dflash_stack_add_rmsnorm(s->resid, pd.delta, weight, out, d.block, d.hidden, d.eps, st);
}

int qmm(dflash_stack* s, const dflash_bf16* x, const dflash_qweight& q, dflash_bf16* y, cudaStream_t st) {
    return dflash_qmm(x, q.w, q.scales, q.biases, y, s->d.block, q.N, q.K, s->d.group, s->d.bits, s->ws, s->ws_bytes,
                      st);
}

// A row-sharded projection whose output is summed over the ranks: pushed into every rank's
// exchange set (world > 1) or written to `delta` (world 1).
int qmm_reduced(dflash_stack* s, const dflash_bf16* x, const dflash_qweight& q, bool swiglu, cudaStream_t st,
                Pending* pd) {
    const dflash_stack_desc& d = s->d;
    dflash_qmm_options o = {};
    o.x_swiglu = swiglu ? 1 : 0;
    o.world = 1;
    if (d.world > 1) {
        o.push = 1;
        o.rank = d.rank;
        o.world = d.world;
        o.set = s->set;
        o.bases = d.exchange;
        if (int r = dflash_qmm_ex(x, q.w, q.scales, q.biases, nullptr, d.block, q.N, q.K, d.group, d.bits, s->ws,
                                  s->ws_bytes, &o, st))
            return r;
        *pd = Pending{nullptr, s->set};
        s->set ^= 1;
        return DFLASH_OK;
    }
    if (int r = dflash_qmm_ex(x, q.w, q.scales, q.biases, s->delta, d.block, q.N, q.K, d.group, d.bits, s->ws,
                              s->ws_bytes, &o, st))
        return r;
    *pd = Pending{s->delta, -1};
    return DFLASH_OK;
}

int gdn_layer(dflash_stack* s, const dflash_stack_layer& L, int gi, cudaStream_t st, Pending* pd) {
    const dflash_stack_desc& d = s->d;
    const int M = d.block, h = d.gdn_heads, hk = d.gdn_key_heads, dk = d.gdn_dk, dv = d.gdn_dv, ni = n_in(d);
    dflash_bf16* proj = s->proj[gi];
    if (int r = qmm(s, s->normed, L.in_proj, proj, st)) return r;
    dflash_bf16* q = s->cqkv[gi];
    dflash_bf16* k = q + (size_t)M * hk * dk;
    dflash_bf16* v = k + (size_t)M * hk * dk;
    const dflash_bf16* ab = proj + 2 * hk * dk + 2 * h * dv;
    int r = hk == h ? dflash_stack_gdn_conv_gates(proj, ni, L.window, L.conv, q, ab, ni, L.a_log, L.dt_bias,
                                                  s->alpha[gi], s->beta[gi], M, h, dk, d.conv_kernel, st)
                    : dflash_stack_gdn_conv_gates_grouped(proj, ni, L.window, L.conv, q, ab, ni, L.a_log, L.dt_bias,
                                                          s->alpha[gi], s->beta[gi], M, h, hk, dk, d.conv_kernel,
                                                          nullptr, st);
    if (r) return r;
    const float qs = 1.0f / std::sqrt((float)dk);
    r = hk == h ? dflash_gdn_step(L.snapshot, s->state_out[gi], q, k, v, s->alpha[gi], s->beta[gi], s->gdn_o, M, h,
                                  dk, dv, qs, st)
                : dflash_gdn_step_grouped(L.snapshot, s->state_out[gi], q, k, v, s->alpha[gi], s->beta[gi], s->gdn_o,
                                          M, h, hk, dk, dv, qs, st);
    if (r) return r;
    const dflash_bf16* z = proj + 2 * hk * dk + h * dv;
    if ((r = dflash_stack_gated_norm(s->gdn_o, z, ni, L.gdn_norm, s->gdn_normed, M, h, dv, d.eps, st))) return r;
    return qmm_reduced(s, s->gdn_normed, L.out_proj, false, st, pd);
}

int attn_layer(dflash_stack* s, const dflash_stack_layer& L, cudaStream_t st, Pending* pd) {
    const dflash_stack_desc& d = s->d;
    const int M = d.block, hq = d.attn_heads, hkv = d.kv_heads, hd = d.head_dim;
    const int ld = (2 * hq + 2 * hkv) * hd;
    if (int r = qmm(s, s->normed, L.qkv, s->qkv, st)) return r;
    if (int r = dflash_stack_attn_prep(s->qkv, ld, L.q_norm, L.k_norm, L.cache_k, L.cache_v, M, hq, hkv, hd,
                                       d.rotary_dim, s->context, d.max_len, d.eps, d.rope_theta, st))
        return r;
    if (int r = dflash_stack_attn_decode(s->qkv, ld, L.cache_k, L.cache_v, s->attn_out, M, hq, hkv, hd, s->context,
                                         d.max_len, 1.0f / std::sqrt((float)hd), st))
        return r;
    return qmm_reduced(s, s->attn_out, L.o_proj, false, st, pd);
}

int forward(dflash_stack* s, const dflash_bf16* hidden, dflash_bf16* out, cudaStream_t st) {
    const dflash_stack_desc& d = s->d;
    if (s->context + d.block > d.max_len)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack: no cache room for a block of %d at context %d (max_len %d)",
                    d.block, s->context, d.max_len);
    DFLASH_CUDA_TRY(cudaMemsetAsync(s->resid, 0, (size_t)d.block * d.hidden * 4, st));
    Pending pd{hidden, -1};
    int gi = 0;
    for (int i = 0; i < d.layers; ++i) {
        const dflash_stack_layer& L = s->layer[i];
        if (int r = norm(s, pd, L.ln, s->normed, st)) return r;
        int r = L.attention ? attn_layer(s, L, st, &pd) : gdn_layer(s, L, gi++, st, &pd);
        if (r) return r;
        if ((r = norm(s, pd, L.post_ln, s->normed, st))) return r;
        if ((r = qmm(s, s->normed, L.gate_up, s->gate_up, st))) return r;
        if ((r = qmm_reduced(s, s->gate_up, L.down, true, st, &pd))) return r;  // SwiGLU inside the down qmm
    }
    return norm(s, pd, d.final_norm, out, st);
}

}  // namespace stackdrv
}  // namespace dflash

extern "C" int dflash_stack_create(const dflash_stack_desc* desc, int context, dflash_stack** out) {
    using namespace dflash;
    using namespace dflash::stackdrv;
    if (!desc || !out || !desc->layer || !desc->final_norm)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_create: null argument");
    *out = nullptr;
    const dflash_stack_desc& d = *desc;
    if (d.layers < 1 || d.hidden < 1 || d.block < 1 || d.block > 16 || d.world < 1 || d.rank < 0 ||
        d.rank >= d.world || d.group < 1 || (d.bits != 4 && d.bits != 8))
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_create: bad layers/hidden/block/rank/world/format");
    if (d.world > 1 && (!d.exchange || !d.key_exchange))
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_create: world > 1 needs both exchange base arrays");
    if (context < 0 || context + d.block > d.max_len)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_create: context %d + block %d past max_len %d",
                    context, d.block, d.max_len);
    int n_gdn = 0, n_attn = 0;
    for (int i = 0; i < d.layers; ++i) (d.layer[i].attention ? n_attn : n_gdn) += 1;
    if (n_gdn && (d.gdn_heads < 1 || d.gdn_key_heads < 1 || d.gdn_heads % d.gdn_key_heads || d.gdn_dk != d.gdn_dv ||
                  d.conv_kernel < 2))
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_create: bad gated-delta heads/dims/conv kernel");
    if (n_attn && (d.attn_heads < 1 || d.kv_heads < 1 || d.head_dim < 1 || d.rotary_dim < 0))
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_create: bad attention heads/dims");
    // every projection has the shape this rank's shard implies
    const int M = d.block, H = d.hidden;
    int inter = -1;
    for (int i = 0; i < d.layers; ++i) {
        const dflash_stack_layer& L = d.layer[i];
        if (!L.ln || !L.post_ln) return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_create: layer %d norms", i);
        if (L.attention) {
            const int nq = (2 * d.attn_heads + 2 * d.kv_heads) * d.head_dim;
            if (!quant_ok(L.qkv, nq, H) || !quant_ok(L.o_proj, H, d.attn_heads * d.head_dim) || !L.q_norm ||
                !L.k_norm || !L.cache_k || !L.cache_v)
                return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_create: attention layer %d tensors", i);
        } else {
            if (!quant_ok(L.in_proj, n_in(d), H) || !quant_ok(L.out_proj, H, d.gdn_heads * d.gdn_dv) || !L.conv ||
                !L.a_log || !L.dt_bias || !L.gdn_norm || !L.snapshot || !L.window)
                return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_create: gated-delta layer %d tensors", i);
        }
        if (inter < 0) inter = L.down.K;
        if (!quant_ok(L.gate_up, 2 * inter, H) || !quant_ok(L.down, H, inter))
            return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_create: MLP of layer %d", i);
    }
    if (!quant_ok(d.lm_head, d.lm_head.N, H) || d.lm_head.N < 1 || d.vocab0 < 0)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_create: LM head");

    dflash_stack* s = new (std::nothrow) dflash_stack();
    if (!s) return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_create: out of host memory");
    s->d = d;
    s->layer.assign(d.layer, d.layer + d.layers);
    s->d.layer = s->layer.data();
    s->context = context;
    auto cleanup = [&](int st) {
        dflash_stack_destroy(s);
        return st;
    };
    int st;
    const int hq = d.attn_heads, hkv = d.kv_heads, hd = d.head_dim;
    const int h = d.gdn_heads, dk = d.gdn_dk, dv = d.gdn_dv;
    if ((st = alloc(s, &s->resid, (size_t)M * H)) || (st = alloc(s, &s->normed, (size_t)M * H)) ||
        (st = alloc(s, &s->delta, (size_t)M * H)) || (st = alloc(s, &s->out, (size_t)M * H)) ||
        (st = alloc(s, &s->keys, (size_t)M)) || (st = alloc(s, &s->gate_up, (size_t)M * 2 * inter)))
        return cleanup(st);
    if (n_attn && ((st = alloc(s, &s->qkv, (size_t)M * (2 * hq + 2 * hkv) * hd)) ||
                   (st = alloc(s, &s->attn_out, (size_t)M * hq * hd))))
        return cleanup(st);
    if (n_gdn) {
        const int C = conv_channels(d);
        if ((st = alloc(s, &s->gdn_o, (size_t)M * h * dv)) || (st = alloc(s, &s->gdn_normed, (size_t)M * h * dv)) ||
            (st = alloc(s, &s->conv_in, (size_t)M * C)) || (st = alloc(s, &s->window_tmp, (size_t)(d.conv_kernel - 1) * C)))
            return cleanup(st);
        s->proj.resize(n_gdn);
        s->cqkv.resize(n_gdn);
        s->alpha.resize(n_gdn);
        s->beta.resize(n_gdn);
        s->state_out.resize(n_gdn);
        for (int g = 0; g < n_gdn; ++g)
            if ((st = alloc(s, &s->proj[g], (size_t)M * n_in(d))) || (st = alloc(s, &s->cqkv[g], (size_t)M * C)) ||
                (st = alloc(s, &s->alpha[g], (size_t)M * h)) || (st = alloc(s, &s->beta[g], (size_t)M * h)) ||
                (st = alloc(s, &s->state_out[g], (size_t)h * dv * dk)))
                return cleanup(st);
    }
    // one qmm workspace for every projection (its size grows with M and K only)
    size_t need = dflash_qmm_workspace_bytes(M, d.lm_head.N, H, d.group, d.bits);
    auto upd = [&](const dflash_qweight& q) {
        if (q.w) need = std::max(need, dflash_qmm_workspace_bytes(M, q.N, q.K, d.group, d.bits));
    };
    for (const auto& L : s->layer) {
        upd(L.in_proj);
        upd(L.out_proj);
        upd(L.qkv);
        upd(L.o_proj);
        upd(L.gate_up);
        upd(L.down);
    }
    s->ws_bytes = need;
    if (need) {
        uint8_t* w = nullptr;
        if ((st = alloc(s, &w, need))) return cleanup(st);
        s->ws = w;
    }
    *out = s;
    return DFLASH_OK;
}

extern "C" int dflash_stack_forward(dflash_stack* s, const dflash_bf16* hidden, dflash_bf16* out,
                                    dflash_stream_t stream) {
    using namespace dflash;
    if (!s || !hidden) return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_forward: null argument");
    return stackdrv::forward(s, hidden, out ? out : s->out, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int dflash_stack_verify(dflash_stack* s, const dflash_bf16* hidden, const int32_t* proposals,
                                   int32_t* target_tokens, int32_t* accepted, dflash_stream_t stream) {
    using namespace dflash;
    if (!s || !hidden || !proposals || !target_tokens || !accepted)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_verify: null argument");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const dflash_stack_desc& d = s->d;
    if (int r = stackdrv::forward(s, hidden, s->out, st)) return r;
    // the LM head of this rank's vocabulary shard, reduced to argmax keys in its epilogue
    dflash_qmm_options o = {};
    o.world = 1;
    o.argmax_keys = s->keys;
    o.argmax_index_base = d.vocab0;
    if (int r = dflash_qmm_ex(s->out, d.lm_head.w, d.lm_head.scales, d.lm_head.biases, nullptr, d.block, d.lm_head.N,
                              d.hidden, d.group, d.bits, s->ws, s->ws_bytes, &o, st))
        return r;
    if (d.world > 1) {
        // one key exchange per round (the layers' all-reduces keep the ranks in step), set 0
        if (int r = dflash_tp_push(reinterpret_cast<const dflash_bf16*>(s->keys), d.key_exchange, d.rank, d.world,
                                   d.block, 4, 0, st))
            return r;
        return dflash_accept_reduce(d.key_exchange[d.rank], d.world, 0, proposals, d.block - 1, target_tokens,
                                    accepted, st);
    }
    return dflash_accept(s->keys, proposals, d.block - 1, target_tokens, accepted, st);
}

extern "C" int dflash_stack_commit(dflash_stack* s, const int32_t* rows, int keep, dflash_stream_t stream) {
    using namespace dflash;
    if (!s) return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_commit: null stack");
    const dflash_stack_desc& d = s->d;
    if (keep < 1 || keep > d.block)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_commit: keep %d outside 1..%d", keep, d.block);
    for (int i = 0; i < keep; ++i)  // chain rounds: the accepted rows are the block's first keep rows
        if (rows && rows[i] != i)
            return fail(DFLASH_ERR_UNSUPPORTED, "dflash_stack_commit: rows must be 0 .. keep-1 (chain rounds)");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int M = d.block, h = d.gdn_heads, hk = d.gdn_key_heads, dk = d.gdn_dk, dv = d.gdn_dv;
    const int C = stackdrv::conv_channels(d), ni = stackdrv::n_in(d);
    int gi = 0;
    for (int i = 0; i < d.layers; ++i) {
        const dflash_stack_layer& L = s->layer[i];
        if (L.attention) continue;  // chain rounds: the block's k and v already sit at context .. context+keep-1
        const dflash_bf16* k = s->cqkv[gi] + (size_t)M * hk * dk;
        const dflash_bf16* v = k + (size_t)M * hk * dk;
        // the state after the kept rows, replayed from the snapshot over the capture
        int r = hk == h ? dflash_gdn_replay(L.snapshot, s->state_out[gi], k, v, s->alpha[gi], s->beta[gi], nullptr,
                                            keep, M, 1, h, dk, dv, st)
                        : dflash_gdn_replay_grouped(L.snapshot, s->state_out[gi], k, v, s->alpha[gi], s->beta[gi],
                                                    nullptr, keep, M, 1, h, hk, dk, dv, st);
        if (r) return r;
        DFLASH_CUDA_TRY(cudaMemcpyAsync(L.snapshot, s->state_out[gi], (size_t)h * dv * dk * 4,
                                        cudaMemcpyDeviceToDevice, st));
        // the conv window rebuilt from the kept rows' conv inputs (the in-projection's first C channels)
        DFLASH_CUDA_TRY(cudaMemcpy2DAsync(s->conv_in, (size_t)C * 2, s->proj[gi], (size_t)ni * 2, (size_t)C * 2, M,
                                          cudaMemcpyDeviceToDevice, st));
        if ((r = dflash_gdn_conv_rollback(L.window, s->window_tmp, s->conv_in, nullptr, keep, M, 1, d.conv_kernel - 1, C,
                                          st)))
            return r;
        DFLASH_CUDA_TRY(cudaMemcpyAsync(L.window, s->window_tmp, (size_t)(d.conv_kernel - 1) * C * 2,
                                        cudaMemcpyDeviceToDevice, st));
        ++gi;
    }
    return DFLASH_OK;
}

extern "C" int dflash_stack_advance(dflash_stack* s, int n) {
    using namespace dflash;
    if (!s) return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_advance: null stack");
    if (n < 0 || s->context + n > s->d.max_len)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_advance: context %d + %d past max_len %d", s->context,
                    n, s->d.max_len);
    s->context += n;
    return DFLASH_OK;
}

extern "C" int dflash_stack_context(const dflash_stack* s) { return s ? s->context : -1; }

extern "C" const dflash_bf16* dflash_stack_output(const dflash_stack* s) { return s ? s->out : nullptr; }

extern "C" void dflash_stack_destroy(dflash_stack* s) {
    if (!s) return;
    for (void* p : s->allocations) cudaFree(p);
    delete s;
}
