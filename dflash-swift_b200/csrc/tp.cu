// Tensor-parallel exchange over peer memory (NVLink / NVSwitch), for the all-reduce after
// the row-sharded projections of the verify stack.
//
// Every rank owns one exchange buffer (cudaMalloc, shared with the other ranks of the
// node through CUDA IPC).  Layout, identical on every rank:
//   flags [2][kMaxRanks] u32   flag[b][r]: CTAs of rank r's pushes into this buffer's slot
//                              set b (monotonic, never reset)
//   seq   [2] u32              this rank's own pushes into set b (monotonic)
//   data  [2][world][M_max H]  set b, slot r: rank r's bf16 partial
// A push (dflash_tp_push) stores this rank's partial into slot `rank` of set b of every
// rank's buffer (own included) with plain vector stores over NVLink, then each CTA
// releases a system-scope increment of the flag of every destination.  The consumer
// (dflash_stack_add_rmsnorm_reduce) waits, bounded, until every source's flag has
// reached seq[b] x push CTAs, and sums the slots in rank order, so every rank computes
// the same bits.  Calls alternate b = 0, 1: a rank can only push into set b again after
// it has consumed the other set's exchange, which every peer pushed only after it had
// consumed set b; so two sets suffice and no slot is overwritten while it is read.
#include <cstring>

#include "common.cuh"
#include "dflash_stack.h"

namespace dflash {
namespace tp {

constexpr int kMaxRanks = 8;
constexpr int kPushBlocks = 32;       // CTAs of a push; flags count CTAs
constexpr size_t kHeaderBytes = 256;  // flags + seq, padded

struct Header {
    uint32_t flags[2][kMaxRanks];
    uint32_t seq[2];
};
static_assert(sizeof(Header) <= kHeaderBytes, "header");

__host__ __device__ inline size_t slot_elems(int M, int H) { return (size_t)M * H; }
__host__ __device__ inline size_t exchange_bytes(int world, int M, int H) {
    return kHeaderBytes + 2 * (size_t)world * slot_elems(M, H) * 2;
}
__host__ __device__ inline uint16_t* slot_ptr(void* base, int world, int M, int H, int set, int r) {
    return reinterpret_cast<uint16_t*>(static_cast<uint8_t*>(base) + kHeaderBytes) +
           ((size_t)set * world + r) * slot_elems(M, H);
}

struct Bases {
    void* b[kMaxRanks];
};

__device__ __forceinline__ void red_release_sys_add(uint32_t* addr, uint32_t v) {
    asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* addr) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
    return v;
}

// part: bf16 [M, H] (16-byte aligned, M H a multiple of 8).  Each CTA stores a contiguous
// share of the 16-byte chunks into every destination, then bumps their flags.
__global__ void __launch_bounds__(256) push_kernel(const uint4* __restrict__ part, Bases bases, int rank, int world,
                                                   int M, int H, int set) {
    pdl_wait();
    pdl_launch_dependents();
    const size_t chunks = slot_elems(M, H) / 8;
    const size_t per = (chunks + gridDim.x - 1) / gridDim.x;
    const size_t c0 = per * blockIdx.x, c1 = c0 + per < chunks ? c0 + per : chunks;
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        Header* own = reinterpret_cast<Header*>(bases.b[rank]);
        own->seq[set] += 1;  // read by this rank's consumer, which runs after this kernel
    }
    for (int r = 0; r < world; ++r) {
        uint4* dst = reinterpret_cast<uint4*>(slot_ptr(bases.b[r], world, M, H, set, rank));
        for (size_t c = c0 + threadIdx.x; c < c1; c += blockDim.x) dst[c] = part[c];
    }
    __syncthreads();  // every store of this CTA is issued before the flags move
    if (threadIdx.x < world) {
        __threadfence_system();
        Header* h = reinterpret_cast<Header*>(bases.b[threadIdx.x]);
        red_release_sys_add(&h->flags[set][rank], 1u);
    }
}

// Bounded wait (about a second) until every source's flag of `set` has reached the
// expected count; false after a timeout (the device error word records it).
__device__ __forceinline__ bool wait_flags(const Header* h, int world, int set, uint32_t expect) {
    for (int r = 0; r < world; ++r) {
        if (ld_acquire_sys(&h->flags[set][r]) >= expect) continue;
        const unsigned long long t0 = globaltimer_ns();
        while (ld_acquire_sys(&h->flags[set][r]) < expect) {
            if (globaltimer_ns() - t0 > kWaitLimitNs) {
                atomicOr(&g_device_error, DFLASH_DEVERR_ALLREDUCE);
                return false;
            }
            __nanosleep(64);
        }
    }
    return true;
}

}  // namespace tp
}  // namespace dflash

using namespace dflash;

extern "C" size_t dflash_tp_exchange_bytes(int world, int M, int H) {
    if (world < 1 || world > tp::kMaxRanks || M < 1 || H < 1) return 0;
    return tp::exchange_bytes(world, M, H);
}

extern "C" int dflash_tp_exchange_alloc(size_t bytes, void** ptr) {
    if (!ptr || bytes < tp::kHeaderBytes) return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_tp_exchange_alloc: bad arguments");
    *ptr = nullptr;
    void* p = nullptr;
    DFLASH_CUDA_TRY(cudaMalloc(&p, bytes));
    const cudaError_t e = cudaMemset(p, 0, bytes);
    if (e != cudaSuccess) {
        cudaFree(p);
        return fail(DFLASH_ERR_CUDA, "cudaMemset(exchange): %s", cudaGetErrorString(e));
    }
    DFLASH_CUDA_TRY(cudaDeviceSynchronize());
    *ptr = p;
    return DFLASH_OK;
}

extern "C" int dflash_tp_exchange_free(void* ptr) {
    if (ptr) DFLASH_CUDA_TRY(cudaFree(ptr));
    return DFLASH_OK;
}

extern "C" int dflash_ipc_get_handle(const void* ptr, void* handle) {
    if (!ptr || !handle) return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_ipc_get_handle: bad arguments");
    cudaIpcMemHandle_t h;
    DFLASH_CUDA_TRY(cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)));
    memcpy(handle, &h, sizeof(h));
    return DFLASH_OK;
}

extern "C" int dflash_ipc_open_handle(const void* handle, void** ptr) {
    if (!ptr || !handle) return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_ipc_open_handle: bad arguments");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    *ptr = nullptr;
    DFLASH_CUDA_TRY(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
    return DFLASH_OK;
}

extern "C" int dflash_ipc_close_handle(void* ptr) {
    if (ptr) DFLASH_CUDA_TRY(cudaIpcCloseMemHandle(ptr));
    return DFLASH_OK;
}

extern "C" int dflash_tp_push(const dflash_bf16* part, void* const* bases, int rank, int world, int M, int H, int set,
                              dflash_stream_t stream) {
    if (!part || !bases || world < 1 || world > tp::kMaxRanks || rank < 0 || rank >= world || M < 1 || H < 1 ||
        (set != 0 && set != 1))
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_tp_push: bad arguments");
    if (((size_t)M * H) % 8 || !aligned16(part))
        return fail(DFLASH_ERR_MISALIGNED, "dflash_tp_push: the partial must be 16-byte aligned with M H a multiple of 8");
    tp::Bases b = {};
    for (int r = 0; r < world; ++r) {
        if (!bases[r] || !aligned16(bases[r])) return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_tp_push: bad base %d", r);
        b.b[r] = bases[r];
    }
    DFLASH_CUDA_TRY(launch_chained(tp::push_kernel, dim3(tp::kPushBlocks), dim3(256), 0,
                                   reinterpret_cast<cudaStream_t>(stream), 1, reinterpret_cast<const uint4*>(part), b,
                                   rank, world, M, H, set));
    return DFLASH_OK;
}
