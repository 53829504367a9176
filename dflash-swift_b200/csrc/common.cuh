// Shared device/host helpers for libdflashcuda: status handling, bf16 bit helpers,
// mbarrier + TMA (cp.async.bulk.tensor) PTX wrappers with bounded waits, and the
// tensor-map encoder obtained from the driver at run time (no -lcuda link, so the
// library loads on hosts without a GPU driver).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>

#include "dflash_cuda.h"

namespace dflash {

// ---------------------------------------------------------------- host status
void set_last_error(const char* fmt, ...);
int fail(int status, const char* fmt, ...);

#define DFLASH_CUDA_TRY(expr)                                                              \
    do {                                                                                   \
        cudaError_t _e = (expr);                                                           \
        if (_e != cudaSuccess)                                                             \
            return ::dflash::fail(DFLASH_ERR_CUDA, "%s failed: %s", #expr,                  \
                                  cudaGetErrorString(_e));                                 \
    } while (0)

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------- device error word
// Set (atomicOr) by any kernel whose bounded wait ran out; read and cleared through
// dflash_device_error().  Bits: DFLASH_DEVERR_*.
__device__ unsigned int g_device_error;

// Upper bound on any single wait inside a kernel.  Normal waits last microseconds.
constexpr unsigned long long kWaitLimitNs = 1000ull * 1000ull * 1000ull;

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_shared() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\t"
        "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\t"
        "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
        "r"(bytes)
        : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Suspend time asked of a blocking try_wait: the thread sleeps until the phase
// completes or this many nanoseconds pass, instead of spinning.
constexpr uint32_t kSuspendHintNs = 20000;

// try_wait that suspends the thread for up to kSuspendHintNs.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "n"(kSuspendHintNs)
        : "memory");
    return ok != 0;
}

// Waits for the phase with the given parity to complete.  Gives up after
// kWaitLimitNs, records `errbit` in g_device_error and in *abort (shared), and returns
// false.  Returns false at once when *abort is already set.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  volatile int* abort, unsigned errbit) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    const unsigned long long t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait_sleep(bar, parity)) return true;
        if (*abort) return false;
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
            atomicOr(&g_device_error, errbit);
            *abort = 1;
            return false;
        }
    }
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------- misc device
__device__ __forceinline__ uint16_t lds16(uint32_t addr) {
    uint16_t v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(addr));
    return v;
}

// gpu-scope release add (no return value) and acquire load, for cross-CTA hand-offs.
__device__ __forceinline__ void red_release_add(int* addr, int v) {
    asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire(const int* addr) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
    return v;
}

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ float bf16_bits_to_float(uint16_t b) {
    return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

// D = A * B + D, m16n8k16, bf16 inputs, fp32 accumulate.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---------------------------------------------------------------- speculative tree rows
// A tree round's block rows carry a parent list in device memory: parents[0] = -1 (the
// anchor) and parents[r] in [0, r) for r > 0, so every path from the anchor visits rows
// in increasing order.  Tree rounds have at most kMaxTreeRows rows, so a set of rows is
// one 32-bit mask.
constexpr int kMaxTreeRows = 32;

// parents[r] when it names an earlier row, else -1: a malformed list makes a row its own
// root instead of sending any walk out of range.
__device__ __forceinline__ int tree_parent(const int32_t* __restrict__ parents, int r) {
    const int p = r > 0 ? parents[r] : -1;
    return p >= 0 && p < r ? p : -1;
}

struct TreeRow {
    uint32_t path;  // bit a set when row a lies on the anchor-to-row path (the row included)
    int depth;      // parent steps from the row back to its root
};

// The path mask and depth of row t < kMaxTreeRows (at most t + 1 dependent loads).
__device__ __forceinline__ TreeRow tree_walk(const int32_t* __restrict__ parents, int t) {
    TreeRow w{0u, 0};
    int r = t;
    for (int s = 0; s < kMaxTreeRows && r >= 0; ++s) {
        w.path |= 1u << r;
        r = tree_parent(parents, r);
        w.depth += r >= 0;
    }
    return w;
}

// ---------------------------------------------------------------- tensor maps (host)
// Encodes a 2D tiled tensor map: global [rows, cols] row-major with `row_bytes`
// pitch, box [box_rows, box_cols].  Returns DFLASH_OK or an error status.
int encode_tensor_map_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base,
                         uint64_t cols, uint64_t rows, uint64_t row_bytes, uint32_t box_cols,
                         uint32_t box_rows, CUtensorMapSwizzle swizzle);

int sm_count(int device);


// ------------------------------------------------------------------ launch chaining and clusters
// Programmatic dependent launch: a kernel launched with the programmatic-serialization
// attribute may start before its predecessor in the stream has finished; pdl_wait()
// blocks until that predecessor has completed and its memory is visible (a no-op when
// the kernel was launched without the attribute), and pdl_launch_dependents() lets the
// next such kernel start.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_size() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
    return r;
}
// Address of the same shared-memory offset in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t addr, uint32_t rank) {
    uint32_t d;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(addr), "r"(rank));
    return d;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ float ld_shared_cluster_f32(uint32_t cluster_addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(cluster_addr) : "memory");
    return v;
}

// Host: launch `kernel` on `stream` with programmatic dependent launch allowed and, when
// cluster > 1, thread-block clusters of `cluster` CTAs along x.
template <class... KArgs, class... Args>
cudaError_t launch_chained(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                           unsigned cluster, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    int n = 1;
    if (cluster > 1) {
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = cluster;
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        n = 2;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

}  // namespace dflash
