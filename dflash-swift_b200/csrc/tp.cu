// Tensor-parallel exchange over peer memory (NVLink / NVSwitch), for the all-reduce after
// the row-sharded projections of the verify stack.
//
// Every rank owns one exchange buffer (cudaMalloc, shared with the other ranks of the
// node through CUDA IPC).  Layout, identical on every rank:
//   header: seq[2], next[2] u32 (this rank's own bookkeeping, see below)
//   data  [2 sets][world slots][M H / 2] u64 words
// Each data word carries two bf16 of a partial in its low half and the exchange's epoch
// in its high half, written with one 8-byte store, so a reader that sees the epoch it
// expects has the data of that exchange: no fence and no separate flag is needed (the
// scheme of low-latency collective protocols).  A push (dflash_tp_push) writes this
// rank's partial into slot `rank` of set b of every rank's buffer (own included) with
// epoch e = seq[b] + 1 and records next[b] = e; the consumer
// (dflash_stack_add_rmsnorm_reduce) waits, bounded, until every word it reads carries
// e = next[b], sums the slots in rank order (so every rank computes the same bits) and
// records seq[b] = e.  Exchanges alternate b = 0, 1: a rank pushes into set b again only
// after consuming the other set's exchange, which every peer pushed only after it had
// consumed set b; so no slot is overwritten while it is read, and epochs never repeat.
#include <cstring>

#include "common.cuh"
#include "dflash_stack.h"
#include "tp_layout.cuh"

namespace dflash {
namespace tp {

constexpr int kPushBlocks = 128;  // spreads the NVLink stores over many SMs

// part: bf16 [M, H] (4-byte aligned, H even).  Thread i of the grid handles data words
// i, i + grid, ... and writes each to every destination.
__global__ void __launch_bounds__(256) push_kernel(const uint32_t* __restrict__ part, Bases bases, int rank, int world,
                                                   int M, int H, int set) {
    pdl_wait();
    pdl_launch_dependents();
    Header* own = reinterpret_cast<Header*>(bases.b[rank]);
    const uint32_t e = own->seq[set] + 1u;
    if (blockIdx.x == 0 && threadIdx.x == 0) own->next[set] = e;
    const uint64_t hi = (uint64_t)e << 32;
    const size_t words = slot_words(M, H);
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < words; i += (size_t)gridDim.x * blockDim.x) {
        const uint64_t w = hi | part[i];
        for (int r = 0; r < world; ++r) st_relaxed_sys_u64(slot_ptr(bases.b[r], world, M, H, set, rank) + i, w);
    }
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
    if (H % 2 || (reinterpret_cast<uintptr_t>(part) & 3u))
        return fail(DFLASH_ERR_MISALIGNED, "dflash_tp_push: the partial must be 4-byte aligned with H even");
    tp::Bases b = {};
    for (int r = 0; r < world; ++r) {
        if (!bases[r] || !aligned16(bases[r])) return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_tp_push: bad base %d", r);
        b.b[r] = bases[r];
    }
    DFLASH_CUDA_TRY(launch_chained(tp::push_kernel, dim3(tp::kPushBlocks), dim3(256), 0,
                                   reinterpret_cast<cudaStream_t>(stream), 1, reinterpret_cast<const uint32_t*>(part),
                                   b, rank, world, M, H, set));
    return DFLASH_OK;
}
