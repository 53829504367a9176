/*
 * CPU oracle for the gated-delta recurrence capture/replay (TEST INFRASTRUCTURE ONLY).
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU legs may load this file's
 * library; libdflashcuda.so never links or calls it.
 *
 * The reference's recurrence lives in the un-vendored random1st/mlx-swift-lm fork
 * (branch dflash-multilayer-tap, rev 58f641eb); its call sites are
 * Sources/DFlashKit/DFlashSpeculativeGenerator.swift:391-393 (capture requested),
 * :450-461 (rollbackGatedDeltaRound / rollbackGatedDeltaTree) and its contract is
 * Tests/DFlashKitTests/GatedDeltaRollbackTests.swift:84-111 (rolled-back caches equal a
 * committed forward over the kept positions) and SpeculativeTreeTests.swift:170-225
 * (scattered keepRows).  The per-step arithmetic restated here is the published gated
 * delta rule in the decay-first form used by MLX's gated-delta ops:
 *
 *     S   <- alpha_t * S                      (S is [dv, dk] per head, fp32 in the cache)
 *     u   <- v_t - S k_t                      (dv)
 *     S   <- S + beta_t * u k_t^T
 *     o_t <- S q_t                            (output of the step, after the update)
 *
 * Parity status: the fork's exact gate parametrisation (how alpha and beta come from the
 * layer's projections) is not in the reference tree, so it is UNPINNED; the replay
 * contract takes alpha and beta as captured inputs and does not depend on it.  The
 * defining property replay(keep) == committed forward(keep) is what the tests pin.
 *
 * Layouts (one layer): state [H, dv, dk] fp32; q, k [T, H, dk] bf16; v [T, H, dv] bf16;
 * alpha, beta [T, H] fp32; o [T, H, dv].  Computation is in fp64.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static inline double bf(uint16_t h) {
    uint32_t u = ((uint32_t)h) << 16;
    float f;
    memcpy(&f, &u, 4);
    return (double)f;
}

/*
 * Runs the recurrence for one layer over the positions rows[0..n_rows-1] (or
 * 0..n_rows-1 when rows == NULL) from state s0.  Writes the final state (fp64) and,
 * when q and o are given, the per-position outputs o (fp64, [n_rows, H, dv]).
 */
void oracle_gdn_recurrence(const float* s0, const uint16_t* q, const uint16_t* k,
                           const uint16_t* v, const float* alpha, const float* beta,
                           const int32_t* rows, int n_rows, int H, int dk, int dv, double q_scale,
                           double* s_out, double* o) {
    const size_t per_head = (size_t)dv * dk;
    double* u = (double*)malloc(sizeof(double) * dv);
    double* kk = (double*)malloc(sizeof(double) * dk);
    double* qq = (double*)malloc(sizeof(double) * dk);
    for (int h = 0; h < H; ++h) {
        double* S = s_out + (size_t)h * per_head;
        for (size_t i = 0; i < per_head; ++i) S[i] = (double)s0[(size_t)h * per_head + i];
        for (int r = 0; r < n_rows; ++r) {
            const int t = rows ? rows[r] : r;
            const double a = (double)alpha[(size_t)t * H + h];
            const double b = (double)beta[(size_t)t * H + h];
            for (int j = 0; j < dk; ++j) kk[j] = bf(k[((size_t)t * H + h) * dk + j]);
            for (size_t i = 0; i < per_head; ++i) S[i] *= a;
            for (int i = 0; i < dv; ++i) {
                double dot = 0.0;
                for (int j = 0; j < dk; ++j) dot += S[(size_t)i * dk + j] * kk[j];
                u[i] = bf(v[((size_t)t * H + h) * dv + i]) - dot;
            }
            for (int i = 0; i < dv; ++i) {
                const double bu = b * u[i];
                for (int j = 0; j < dk; ++j) S[(size_t)i * dk + j] += bu * kk[j];
            }
            if (q && o) {
                for (int j = 0; j < dk; ++j) qq[j] = bf(q[((size_t)t * H + h) * dk + j]) * q_scale;
                for (int i = 0; i < dv; ++i) {
                    double dot = 0.0;
                    for (int j = 0; j < dk; ++j) dot += S[(size_t)i * dk + j] * qq[j];
                    o[((size_t)r * H + h) * dv + i] = dot;
                }
            }
        }
    }
    free(u);
    free(kk);
    free(qq);
}

/*
 * Conv-window rebuild after a rollback: the depthwise causal conv keeps the last
 * (kc-1) conv inputs.  New window = last (kc-1) rows of
 * [window (kc-1 rows) || conv_in[rows[0..n_rows-1]]].  Layout [rows, C], bf16 bits
 * copied verbatim (the rebuild is a pure gather, bit-exact by construction).
 */
void oracle_conv_window(const uint16_t* window, const uint16_t* conv_in, const int32_t* rows,
                        int n_rows, int kc1, int C, uint16_t* out) {
    for (int r = 0; r < kc1; ++r) {
        /* position of output row r in the concatenated sequence of kc1 + n_rows rows */
        const int pos = n_rows + r;
        const uint16_t* src;
        if (pos < kc1) {
            src = window + (size_t)pos * C;
        } else {
            const int j = pos - kc1;
            const int t = rows ? rows[j] : j;
            src = conv_in + (size_t)t * C;
        }
        memcpy(out + (size_t)r * C, src, sizeof(uint16_t) * (size_t)C);
    }
}
