// CPU stand-ins for the Metal Shading Language constructs used by the reference's
// small-M kernel body (Sources/DFlashKit/SmallMQuantizedMatmul.swift:80-165).
// TEST INFRASTRUCTURE ONLY: lets the reference's own kernel text run on host cores so
// the oracle can be checked against it.  Nothing here is shipped.
//
// Execution model emulated: one threadgroup of 256 threads at a time, each thread a
// real OS thread; simdgroup_barrier synchronises the 32 threads of one simdgroup,
// threadgroup_barrier all 256.  A simdgroup_matrix is held whole by every lane (each
// lane computes the full 8x8 product; only lane 0 stores), which gives the same values
// as a distributed fragment.  Products of two bf16 values are exact in fp32, so the
// 8-term fp32 accumulation inside simdgroup_multiply_accumulate is done in k order with
// fmaf; the hardware's internal order is not observable from the reference tree.
#pragma once
#include <barrier>
#include <cstdint>
#include <cstring>
#include <cmath>

typedef unsigned int uint;

struct uint3 {
    uint x, y, z;
};

struct bfloat16_t {
    uint16_t bits;
    bfloat16_t() = default;
    bfloat16_t(float f) {
        uint32_t u;
        std::memcpy(&u, &f, 4);
        if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) {
            bits = (uint16_t)((u >> 16) | 0x40u);
        } else {
            u += 0x7fffu + ((u >> 16) & 1u);
            bits = (uint16_t)(u >> 16);
        }
    }
    operator float() const {
        uint32_t u = ((uint32_t)bits) << 16;
        float f;
        std::memcpy(&f, &u, 4);
        return f;
    }
};

namespace mem_flags {
enum flag { mem_none = 0, mem_threadgroup = 1, mem_device = 2 };
}

struct ShimThreadContext {
    int lane = 0;
    std::barrier<>* simd_bar = nullptr;
    std::barrier<>* tg_bar = nullptr;
};
extern thread_local ShimThreadContext shim_ctx;

inline void simdgroup_barrier(mem_flags::flag) { shim_ctx.simd_bar->arrive_and_wait(); }
inline void threadgroup_barrier(mem_flags::flag) { shim_ctx.tg_bar->arrive_and_wait(); }

template <typename T, int R, int C>
struct simdgroup_matrix {
    T v[R * C];
    simdgroup_matrix() = default;
    // Metal: constructing from a scalar puts it on the diagonal, zero elsewhere.
    explicit simdgroup_matrix(T d) {
        for (int i = 0; i < R; ++i)
            for (int j = 0; j < C; ++j) v[i * C + j] = (i == j) ? d : T(0.0f);
    }
};

template <typename T, int R, int C, typename P>
inline void simdgroup_load(simdgroup_matrix<T, R, C>& m, const P* src, long elements_per_row) {
    for (int i = 0; i < R; ++i)
        for (int j = 0; j < C; ++j) m.v[i * C + j] = T((float)src[i * elements_per_row + j]);
}

template <typename T, int R, int C, typename P>
inline void simdgroup_store(const simdgroup_matrix<T, R, C>& m, P* dst, long elements_per_row) {
    if (shim_ctx.lane != 0) return;
    for (int i = 0; i < R; ++i)
        for (int j = 0; j < C; ++j) dst[i * elements_per_row + j] = P(m.v[i * C + j]);
}

template <int R, int K, int C, typename TA, typename TB>
inline void simdgroup_multiply_accumulate(simdgroup_matrix<float, R, C>& d,
                                          const simdgroup_matrix<TA, R, K>& a,
                                          const simdgroup_matrix<TB, K, C>& b,
                                          const simdgroup_matrix<float, R, C>& c) {
    simdgroup_matrix<float, R, C> r;
    for (int i = 0; i < R; ++i)
        for (int j = 0; j < C; ++j) {
            float acc = c.v[i * C + j];
            for (int k = 0; k < K; ++k) acc = std::fmaf((float)a.v[i * K + k], (float)b.v[k * C + j], acc);
            r.v[i * C + j] = acc;
        }
    d = r;
}
