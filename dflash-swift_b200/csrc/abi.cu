// C-ABI plumbing for libdflashcuda: thread-local error text, status strings, the
// device error word, the run-time resolved tensor-map encoder and a cached SM count.
#include "common.cuh"

namespace dflash {

namespace {
thread_local std::string g_last_error;
}

void set_last_error(const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
}

int fail(int status, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return status;
}

namespace {
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
std::once_flag g_encode_once;
EncodeTiledFn g_encode = nullptr;
cudaError_t g_encode_err = cudaSuccess;
}  // namespace

int encode_tensor_map_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t cols,
                         uint64_t rows, uint64_t row_bytes, uint32_t box_cols, uint32_t box_rows,
                         CUtensorMapSwizzle swizzle) {
    std::call_once(g_encode_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        g_encode_err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
        if (g_encode_err == cudaSuccess && q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    });
    if (!g_encode)
        return fail(DFLASH_ERR_CUDA, "cuTensorMapEncodeTiled unavailable: %s", cudaGetErrorString(g_encode_err));
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = g_encode(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                                CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(DFLASH_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d): dims %llu x %llu pitch %llu box %u x %u",
                    (int)r, (unsigned long long)cols, (unsigned long long)rows, (unsigned long long)row_bytes,
                    box_cols, box_rows);
    return DFLASH_OK;
}

int sm_count(int device) {
    static std::mutex mu;
    static int cached[64] = {0};
    std::lock_guard<std::mutex> lock(mu);
    if (device < 0 || device >= 64) return 1;
    if (!cached[device]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n < 1) n = 1;
        cached[device] = n;
    }
    return cached[device];
}

}  // namespace dflash

extern "C" int dflash_version(void) { return DFLASH_VERSION; }

extern "C" const char* dflash_last_error(void) { return dflash::g_last_error.c_str(); }

extern "C" const char* dflash_status_string(int status) {
    switch (status) {
        case DFLASH_OK: return "ok";
        case DFLASH_ERR_INVALID_ARGUMENT: return "invalid argument";
        case DFLASH_ERR_UNSUPPORTED: return "unsupported shape or format";
        case DFLASH_ERR_MISALIGNED: return "misaligned pointer";
        case DFLASH_ERR_CUDA: return "CUDA error";
        case DFLASH_ERR_NCCL: return "NCCL error";
        case DFLASH_ERR_TIMEOUT: return "device wait timed out";
        case DFLASH_ERR_WORKSPACE: return "workspace missing or too small";
    }
    return "unknown status";
}

extern "C" int dflash_device_error(uint32_t* bits, dflash_stream_t stream) {
    using namespace dflash;
    if (!bits) return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_device_error: null output");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    unsigned int v = 0;
    const unsigned int zero = 0;
    DFLASH_CUDA_TRY(cudaMemcpyFromSymbolAsync(&v, g_device_error, sizeof(v), 0, cudaMemcpyDeviceToHost, st));
    DFLASH_CUDA_TRY(cudaMemcpyToSymbolAsync(g_device_error, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, st));
    DFLASH_CUDA_TRY(cudaStreamSynchronize(st));
    *bits = v;
    return DFLASH_OK;
}
