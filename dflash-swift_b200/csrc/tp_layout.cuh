// Layout of the tensor-parallel exchange buffer shared by the push (tp.cu, and the qmm
// kernel's pushing epilogue) and the reducing RMSNorm (stack.cu).  See tp.cu.
#pragma once

#include "common.cuh"

namespace dflash {
namespace tp {

constexpr int kMaxRanks = 8;
constexpr size_t kHeaderBytes = 256;

struct Header {
    uint32_t seq[2];   // epoch of the last exchange consumed in set b
    uint32_t next[2];  // epoch of the exchange pushed into set b, not yet consumed
};
static_assert(sizeof(Header) <= kHeaderBytes, "header");

__host__ __device__ inline size_t slot_words(int M, int H) { return (size_t)M * H / 2; }
__host__ __device__ inline size_t exchange_bytes(int world, int M, int H) {
    return kHeaderBytes + 2 * (size_t)world * slot_words(M, H) * 8;
}
__host__ __device__ inline uint64_t* slot_ptr(void* base, int world, int M, int H, int set, int r) {
    return reinterpret_cast<uint64_t*>(static_cast<uint8_t*>(base) + kHeaderBytes) +
           ((size_t)set * world + r) * slot_words(M, H);
}

struct Bases {
    void* b[kMaxRanks];
};

__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t* addr, uint64_t v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(addr), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t* addr) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(addr) : "memory");
    return v;
}

// The data word `i` of source r's slot, once it carries epoch e (bounded wait, about a
// second; after a timeout the device error word records it and 0 is returned).  Once an
// exchange has timed out the ranks are out of step, so later waits give up at once
// instead of each spending its second: the host reads the error word and stops.
__device__ __forceinline__ uint32_t wait_word(const uint64_t* p, uint32_t e) {
    uint64_t v = ld_relaxed_sys_u64(p);
    if ((uint32_t)(v >> 32) == e) return (uint32_t)v;
    if (*reinterpret_cast<volatile unsigned int*>(&g_device_error) & DFLASH_DEVERR_ALLREDUCE) return 0u;
    const unsigned long long t0 = globaltimer_ns();
    while (true) {
        v = ld_relaxed_sys_u64(p);
        if ((uint32_t)(v >> 32) == e) return (uint32_t)v;
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
            atomicOr(&g_device_error, DFLASH_DEVERR_ALLREDUCE);
            return 0u;
        }
        __nanosleep(32);
    }
}

}  // namespace tp
}  // namespace dflash
