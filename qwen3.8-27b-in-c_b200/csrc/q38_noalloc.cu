// q38_noalloc.cu - q38cu_tensor_gemm_q8_k_noalloc: the tiled-layout streaming
// GEMM for callers that cannot allocate device memory.
//
// The regular entry point uses the scratch buffer that q38cu_tensor_upload /
// q38cu_tensor_repack allocate with each tiled tensor.  Some callers cannot
// make that allocation: an engine that hands out device memory only from its
// own pre-planned arena and forbids cudaMalloc after start-up (cudaMalloc and
// cudaFree synchronize the device and stall every stream of a serving
// process), or code that receives a tiled tensor whose weights were placed by
// someone else without a scratch buffer.  This entry point allocates nothing:
// its scratch is the file-scope array below, which every GPU that loads the
// library holds until the process exits.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "../../include/q38cuda.h"
#include "q38_internal.h"

namespace {

// Shared scratch of the no-allocation entry point: tile counters first, then
// the partial sums of row tiles that several CTAs share.  The size is stated in
// the public header as Q38CU_NOALLOC_SCRATCH_BYTES.
static __device__ __align__(256) unsigned char g_noalloc_scratch[Q38CU_NOALLOC_SCRATCH_BYTES];

// Device address of g_noalloc_scratch, looked up once per device.  In host
// code the array's name is only a host-side stand-in, so the address must come
// from cudaGetSymbolAddress with that device current.
constexpr int kMaxDevices = 64;
void *g_scratch_address[kMaxDevices] = {nullptr};
std::mutex g_setup_lock;

// Failures are reported through the library's q38cu_last_error().
int fail(const char *message)
{
    q38::set_last_error(message);
    return 0;
}

int fail_cuda(const char *what, cudaError_t e)
{
    char buffer[256];
    std::snprintf(buffer, sizeof(buffer), "%s: %s", what, cudaGetErrorString(e));
    q38::set_last_error(buffer);
    return 0;
}

// Set-up for the current device (first call on that device only).  The
// address stays valid for the life of the CUDA context: a caller that ends
// the context (cudaDeviceReset) must not call this entry point again in the
// same process.
int scratch_for_current_device(void **address, cudaStream_t stream)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail_cuda("cudaGetDevice", e);
    if (dev < 0 || dev >= kMaxDevices) return fail("device index out of range for the no-allocation scratch");
    std::lock_guard<std::mutex> guard(g_setup_lock);
    if (!g_scratch_address[dev]) {
        // The look-up is not a stream operation and cannot be captured: a
        // first call made while `stream` is being captured is refused with
        // the rule rather than with the capture error it would cause.
        cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
        e = cudaStreamIsCapturing(stream, &capture);
        if (e != cudaSuccess) return fail_cuda("cudaStreamIsCapturing", e);
        if (capture != cudaStreamCaptureStatusNone)
            return fail("the first no-allocation call on a device must come before any stream capture");
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) return fail_cuda("cudaGetSymbolAddress(no-allocation scratch)", e);
        g_scratch_address[dev] = p;
    }
    *address = g_scratch_address[dev];
    return 1;
}

}  // namespace

extern "C" {

int q38cu_tensor_gemm_q8_k_noalloc(float *output, const Q38CuQ8KBlock *input, uint32_t batch_size,
                                   uint64_t input_length, const Q38CuTensor *tensor, void *stream)
{
    if (!output || !input || !batch_size || !tensor) return fail("output, input, batch_size and tensor are required");
    if (tensor->layout != Q38CU_LAYOUT_TILED) return fail("the no-allocation GEMM needs a tensor in the tiled layout");
    if (tensor->n_dims != 2 || tensor->shape[0] != input_length || input_length % 256 || !tensor->data)
        return fail("input length does not match the tensor, or the tensor has no data");
    if ((reinterpret_cast<uintptr_t>(tensor->data) & 15u) != 0) return fail("tensor data must be 16-byte aligned");
    if (tensor->tile_rows == 0 || tensor->tile_rows % 8 || tensor->tile_rows > 256)
        return fail("tiled layout needs tile_rows a multiple of 8 in 8..256");
    if (!q38::superblock_bytes(static_cast<int>(tensor->type)))
        return fail("type has no device streaming kernel");
    if (input_length / 256 > 256 || tensor->shape[1] > 0x7fffffffull)
        return fail("input length above 65536 or too many rows");
    const uint64_t need = input_length / 256 * q38::superblock_bytes(static_cast<int>(tensor->type)) *
                          ((tensor->shape[1] + tensor->tile_rows - 1) / tensor->tile_rows * tensor->tile_rows);
    if (tensor->nbytes < need) return fail("tensor nbytes smaller than its tiled shape requires");

    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int rows = static_cast<int>(tensor->shape[1]);
    const int width = static_cast<int>(input_length);
    const int nb = width / 256;
    void *scratch = nullptr;
    for (uint32_t tok0 = 0; tok0 < batch_size;) {
        q38::StreamPlan plan;
        cudaError_t e = q38::stream_plan(static_cast<int>(tensor->type), rows, width,
                                         static_cast<int>(tensor->tile_rows), static_cast<int>(batch_size - tok0),
                                         &plan);
        if (e != cudaSuccess) return fail_cuda("stream plan", e);
        if (plan.scratch_bytes > Q38CU_NOALLOC_SCRATCH_BYTES) {
            char buffer[256];
            std::snprintf(buffer, sizeof(buffer),
                          "shape needs %llu bytes of scratch; the no-allocation maximum is %llu",
                          static_cast<unsigned long long>(plan.scratch_bytes),
                          static_cast<unsigned long long>(Q38CU_NOALLOC_SCRATCH_BYTES));
            return fail(buffer);
        }
        if (!scratch && !scratch_for_current_device(&scratch, s)) return 0;
        // The array keeps whatever the previous call left; the tile counters
        // must start at zero.
        e = cudaMemsetAsync(scratch, 0, plan.counter_bytes, s);
        if (e != cudaSuccess) return fail_cuda("clearing the no-allocation scratch counters", e);
        q38::StreamLaunch l;
        l.weights = tensor->data;
        l.act = input + static_cast<size_t>(tok0) * nb;
        l.tokens = plan.token_group;
        l.out = output + static_cast<size_t>(tok0) * rows;
        l.scratch = scratch;
        l.dbg_w = nullptr;
        l.dbg_x = nullptr;
        e = q38::launch_stream_gemm(static_cast<int>(tensor->type), plan, l, s);
        if (e != cudaSuccess) return fail_cuda("no-allocation stream gemm launch", e);
        tok0 += static_cast<uint32_t>(plan.token_group);
    }
    return 1;
}

}  // extern "C"
