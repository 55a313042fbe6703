// dav2cuda_linear_int8_noalloc: the int8 linear layer for callers that may
// not allocate device memory. Some host applications own the whole device
// heap — video pipelines, game engines and inference servers that reserve
// their memory at start-up and treat any later cudaMalloc as a failure, or
// run the operator on a real-time path where an allocation (which can
// synchronize the device) is not allowed — so they cannot hand this library
// a per-call workspace. This entry point needs none: its scratch (the int8
// activation codes and row scales, and padded weight rows when K is not a
// multiple of 16) lives in a fixed device array of this library.
//
// Facts a caller relies on:
//  - the scratch is kNoAllocScratchBytes (16 MiB) on every GPU that loads the
//    library, held until the process exits;
//  - problems needing more scratch than that are rejected with
//    DAV2CUDA_INVALID_ARGUMENT before anything is launched;
//  - the first call on a device resolves the array's device address with
//    cudaGetSymbolAddress while that device is current; make that first call
//    before any stream capture. The address is kept for the life of the
//    process: after a cudaDeviceReset (which also frees every buffer the
//    caller passes in) the process must not call this entry point again;
//  - every call on a device shares the one array: calls that overlap on the
//    GPU (different streams, no ordering between them) race on it;
//  - each call overwrites every scratch byte it later reads, so the contents
//    left by an earlier call never leak into a result.
// No cudaMalloc, cudaFree or allocating library routine is called here.
#include <mutex>

#include "kernels.cuh"

namespace {

constexpr uint64_t kNoAllocScratchBytes = 16ull << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint8_t g_linear_int8_scratch[kNoAllocScratchBytes];

std::mutex g_setup_mutex;
void* g_scratch_address[kMaxDevices] = {};

// Device address of the scratch array on the current device (resolved once
// per device; host code must not use the symbol itself as an address).
int scratch_for_current_device(void** out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return dav2cuda::set_error(DAV2CUDA_INTERNAL_ERROR, "linear_int8_noalloc: no current CUDA device");
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_address[dev]) {
        void* p = nullptr;
        const cudaError_t rc = cudaGetSymbolAddress(&p, g_linear_int8_scratch);
        if (rc != cudaSuccess || p == nullptr)
            return dav2cuda::set_error(DAV2CUDA_INTERNAL_ERROR,
                                       "linear_int8_noalloc: cudaGetSymbolAddress of the scratch array failed");
        g_scratch_address[dev] = p;
    }
    *out = g_scratch_address[dev];
    return DAV2CUDA_OK;
}

}  // namespace

extern "C" DAV2CUDA_API uint64_t dav2cuda_linear_int8_noalloc_scratch_limit(void) { return kNoAllocScratchBytes; }

extern "C" DAV2CUDA_API int dav2cuda_linear_int8_noalloc(float* output, const float* input, const uint32_t* int8_weight,
                                            const float* weight_scales, const float* bias, uint32_t rows,
                                            uint32_t input_columns, uint32_t output_columns, uint32_t gelu,
                                            void* stream) {
    if (rows == 0 || input_columns == 0 || output_columns == 0 || input_columns % 4 != 0 ||
        input_columns > 0xFFFFFFF0u)
        return dav2cuda::set_error(DAV2CUDA_INVALID_ARGUMENT, "invalid INT8 linear dimensions");
    const uint64_t need = dav2cuda_linear_int8_workspace_size(rows, input_columns, output_columns);
    if (need > kNoAllocScratchBytes)
        return dav2cuda::set_error(DAV2CUDA_INVALID_ARGUMENT,
                                   "linear_int8_noalloc: this problem needs more scratch than the 16 MiB "
                                   "static array; use dav2cuda_linear_int8 with a caller workspace");
    void* scratch = nullptr;
    if (int rc = scratch_for_current_device(&scratch)) return rc;
    return dav2cuda_linear_int8(output, input, int8_weight, weight_scales, bias, rows, input_columns,
                                output_columns, gelu, scratch, kNoAllocScratchBytes, stream);
}
