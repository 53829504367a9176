// Host-core runner for the reference's small-M Metal kernel text (TEST INFRASTRUCTURE).
//
// build_oracle.py extracts the kernel body that SmallMQuantizedMatmul.source(tiles:)
// assembles (Sources/DFlashKit/SmallMQuantizedMatmul.swift:80-165, with the unpack
// snippet of :55-71 substituted for __UNPACK__ exactly as :183-185 does) into
// oracle/_ref/metal_<bits>_<tiles>.inc, and compiles this file against it.  The only
// textual change made to the reference text is that threadgroup array declarations
// become function-local statics (shared by the 256 threads of the running
// threadgroup).  The dispatch mirrors SmallMQuantizedMatmul.apply (:210-224): grid
// ceil(N/8) threadgroups of 256 threads, template constants KD=K, ND=N, MD=rows, and
// the zero padding of x to 8*tiles rows done by SmallMQuantizedLinear.callAsFunction
// (:271-281).
#include <barrier>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <thread>
#include <vector>

#include "metal_shim.hpp"

thread_local ShimThreadContext shim_ctx;

#define device
#define threadgroup

static void body_4_1(const bfloat16_t* x, const uint* w, const bfloat16_t* sc,
                     const bfloat16_t* bi, bfloat16_t* out, const int KD, const int ND,
                     const int MD, uint3 thread_position_in_threadgroup,
                     uint3 threadgroup_position_in_grid) {
#include "metal_4_1.inc"
}
static void body_4_2(const bfloat16_t* x, const uint* w, const bfloat16_t* sc,
                     const bfloat16_t* bi, bfloat16_t* out, const int KD, const int ND,
                     const int MD, uint3 thread_position_in_threadgroup,
                     uint3 threadgroup_position_in_grid) {
#include "metal_4_2.inc"
}
static void body_8_1(const bfloat16_t* x, const uint* w, const bfloat16_t* sc,
                     const bfloat16_t* bi, bfloat16_t* out, const int KD, const int ND,
                     const int MD, uint3 thread_position_in_threadgroup,
                     uint3 threadgroup_position_in_grid) {
#include "metal_8_1.inc"
}
static void body_8_2(const bfloat16_t* x, const uint* w, const bfloat16_t* sc,
                     const bfloat16_t* bi, bfloat16_t* out, const int KD, const int ND,
                     const int MD, uint3 thread_position_in_threadgroup,
                     uint3 threadgroup_position_in_grid) {
#include "metal_8_2.inc"
}

typedef void (*body_fn)(const bfloat16_t*, const uint*, const bfloat16_t*, const bfloat16_t*,
                        bfloat16_t*, int, int, int, uint3, uint3);

extern "C" {

// Runs the reference kernel on host threads.  x: bf16 bits [rows, K]; w: packed
// [N, K*bits/32]; scales/biases: bf16 bits [N, K/64]; out: bf16 bits [rows, N].
// Returns 0, or -1 for a variant the reference does not build (bits not in {4, 8},
// rows not in 1..16, K not a multiple of 512).
int ref_metal_qmm(const uint16_t* x, const uint32_t* w, const uint16_t* scales,
                  const uint16_t* biases, uint16_t* out, int rows, int N, int K, int bits) {
    if ((bits != 4 && bits != 8) || rows < 1 || rows > 16 || K % 512 != 0 || N < 1) return -1;
    const int tiles = rows <= 8 ? 1 : 2;
    body_fn fn = bits == 4 ? (tiles == 1 ? body_4_1 : body_4_2) : (tiles == 1 ? body_8_1 : body_8_2);
    const int padded = tiles * 8;
    std::vector<bfloat16_t> xp((size_t)padded * K);
    std::memset(xp.data(), 0, sizeof(bfloat16_t) * xp.size());
    std::memcpy(xp.data(), x, sizeof(uint16_t) * (size_t)rows * K);
    const int groups = (N + 7) / 8;
    std::barrier<> tg_bar(256);
    std::vector<std::barrier<>*> simd_bars;
    for (int s = 0; s < 8; ++s) simd_bars.push_back(new std::barrier<>(32));
    std::vector<std::thread> pool;
    for (int tid = 0; tid < 256; ++tid) {
        pool.emplace_back([&, tid]() {
            shim_ctx.lane = tid & 31;
            shim_ctx.simd_bar = simd_bars[tid >> 5];
            shim_ctx.tg_bar = &tg_bar;
            for (int g = 0; g < groups; ++g) {
                fn(xp.data(), (const uint*)w, (const bfloat16_t*)scales,
                   (const bfloat16_t*)biases, (bfloat16_t*)out, K, N, rows,
                   uint3{(uint)tid, 0u, 0u}, uint3{(uint)g, 0u, 0u});
                tg_bar.arrive_and_wait();
            }
        });
    }
    for (auto& t : pool) t.join();
    for (auto* b : simd_bars) delete b;
    return 0;
}
}
