// q38_api.cu - the extern "C" entry points declared in include/q38cuda.h:
// argument validation with the upstream return convention (1 ok, 0 bad
// arguments / unsupported), launch planning and tensor upload.
#include <cmath>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "../../include/q38cuda.h"
#include "q38_gguf_file.h"
#include "q38_internal.h"

namespace {

thread_local char g_error[256] = "";

int fail(const char *fmt, const char *detail = "")
{
    std::snprintf(g_error, sizeof(g_error), fmt, detail);
    return 0;
}

int fail_cuda(const char *what, cudaError_t e)
{
    std::snprintf(g_error, sizeof(g_error), "%s: %s", what, cudaGetErrorString(e));
    return 0;
}

// GGUF block geometry (upstream src/io/qwen38_gguf.c:130-185).
struct Geometry { uint32_t elements, bytes; };

Geometry geometry(uint32_t type)
{
    switch (type) {
    case 0: return {1, 4};       // F32
    case 1: return {1, 2};       // F16
    case 30: return {1, 2};      // BF16
    case 8: return {32, 34};     // Q8_0
    case 20: return {32, 18};    // IQ4_NL
    case 10: return {256, 84};   // Q2_K
    case 11: return {256, 110};  // Q3_K
    case 12: return {256, 144};  // Q4_K
    case 13: return {256, 176};  // Q5_K
    case 14: return {256, 210};  // Q6_K
    case 16: return {256, 66};   // IQ2_XXS
    case 17: return {256, 74};   // IQ2_XS
    case 18: return {256, 98};   // IQ3_XXS
    case 19: return {256, 50};   // IQ1_S
    case 21: return {256, 110};  // IQ3_S
    case 22: return {256, 82};   // IQ2_S
    case 23: return {256, 136};  // IQ4_XS
    case 29: return {256, 56};   // IQ1_M
    default: return {0, 0};
    }
}

// Upstream q38_matrix_type_q8_k (qwen38_model.c:172-182).
bool upstream_q8k_type(uint32_t type)
{
    switch (type) {
    case 10: case 11: case 12: case 13: case 14: case 16: case 17: case 18:
    case 19: case 20: case 21: case 22: case 23: case 29: return true;
    default: return false;
    }
}

// Types the upstream float path accepts (qwen38_quant.c:2768-2810).
bool float_path_type(uint32_t type)
{
    switch (type) {
    case 0: case 1: case 30: case 8: case 10: case 11: case 12: case 13: case 14: case 20: return true;
    default: return false;
    }
}

int env_int(const char *name, int fallback)
{
    const char *v = std::getenv(name);
    return v && *v ? std::atoi(v) : fallback;
}

q38::GemmPlan make_plan(uint32_t type, uint64_t width, uint64_t rows, int batch)
{
    q38::GemmPlan p{};
    p.nb = static_cast<int>(width / 256);
    p.rows = static_cast<int>(rows);
    p.row_bytes = static_cast<uint64_t>(p.nb) * q38::superblock_bytes(static_cast<int>(type));

    // Rows per pass: one superblock per thread; keep >= 95% of the lanes busy
    // with the smallest CTA of at least 128 threads (fall back to best use).
    const int max_threads = batch == 1 ? 384 : 256;  // kernel launch bounds per token tile
    int rho = env_int("Q38CU_ROWS_PER_PASS", 0);
    if (rho <= 0) {
        int best_rho = 1;
        double best_util = -1.0;
        int chosen = 0;
        for (int r = 1; r <= 256; ++r) {
            const int threads = (r * p.nb + 31) / 32 * 32;
            if (threads > max_threads) break;
            const double util = double(r * p.nb) / threads;
            if (!chosen && util >= 0.95 && threads >= 128) chosen = r;
            if (util > best_util + 1e-9) { best_util = util; best_rho = r; }
        }
        rho = chosen ? chosen : best_rho;
    }
    rho = std::max(1, std::min(rho, std::max(1, max_threads / std::max(1, p.nb))));
    if (rho > p.rows) rho = std::max(1, p.rows);
    p.rows_per_pass = rho;
    p.threads = (rho * p.nb + 31) / 32 * 32;

    // Rows per stage: a multiple of rho moving about `target` bytes per copy.
    const uint64_t target = static_cast<uint64_t>(env_int("Q38CU_STAGE_KB", 24)) * 1024;
    const uint64_t pass_bytes = static_cast<uint64_t>(rho) * p.row_bytes;
    uint64_t passes = std::max<uint64_t>(1, (target + pass_bytes / 2) / pass_bytes);
    p.stages = std::max(2, std::min(4, env_int("Q38CU_STAGES", 3)));
    p.max_ctas_per_sm = env_int("Q38CU_CTAS_PER_SM", 0);
    const size_t smem_limit = 227 * 1024;
    for (;;) {
        p.rows_per_stage = static_cast<int>(passes * rho);
        p.stage_bytes = static_cast<uint32_t>((p.rows_per_stage * p.row_bytes + 64 + 15) & ~uint64_t(15));
        if (q38::gemm_smem_for(static_cast<int>(type), p, batch) <= smem_limit) break;
        if (passes > 1) { --passes; continue; }
        if (p.stages > 2) { --p.stages; continue; }
        break;  // a single pass of one row always fits for the supported widths
    }
    p.units = static_cast<int>((rows + p.rows_per_stage - 1) / p.rows_per_stage);
    return p;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

uint64_t rows_padded(uint64_t rows, uint32_t tile_rows)
{
    return (rows + tile_rows - 1) / tile_rows * tile_rows;
}

bool superblock_layout_type(uint32_t type) { return geometry(type).elements == 256; }

int check_matrix(const Q38CuTensor *t, uint64_t input_length)
{
    if (!t) return fail("tensor is NULL%s");
    if (t->n_dims != 2) return fail("tensor must be 2-D%s");
    if (t->shape[0] != input_length) return fail("input length does not match tensor shape[0]%s");
    if (!t->data) return fail("tensor data is NULL%s");
    if (!aligned16(t->data)) return fail("tensor data must be 16-byte aligned%s");
    const Geometry g = geometry(t->type);
    if (!g.elements || input_length % g.elements) return fail("unsupported type or width%s");
    if (t->shape[1] == 0 || t->shape[1] > 0x7fffffffull) return fail("bad row count%s");
    if (t->layout != Q38CU_LAYOUT_GGUF && t->layout != Q38CU_LAYOUT_TILED)
        return fail("unknown tensor layout%s");
    if (t->layout == Q38CU_LAYOUT_TILED && !superblock_layout_type(t->type))
        return fail("tiled layout needs a 256-element block type%s");
    if (t->layout == Q38CU_LAYOUT_TILED && (t->tile_rows == 0 || t->tile_rows % 8 || t->tile_rows > 256))
        return fail("tiled layout needs tile_rows a multiple of 8 in 8..256%s");
    const uint64_t rows = t->layout == Q38CU_LAYOUT_GGUF ? t->shape[1] : rows_padded(t->shape[1], t->tile_rows);
    const uint64_t need = input_length / g.elements * g.bytes * rows;
    if (t->nbytes < need) return fail("tensor nbytes smaller than shape requires%s");
    return 1;
}

uint32_t layout_tile_rows(const Q38CuTensor *t) { return t->layout == Q38CU_LAYOUT_TILED ? t->tile_rows : 0; }

int stream_gemm(float *output, int32_t *w_out, int32_t *x_out, const Q38CuQ8KBlock *input, uint32_t batch,
                uint64_t input_length, const Q38CuTensor *tensor, cudaStream_t stream)
{
    const int rows = static_cast<int>(tensor->shape[1]);
    const int width = static_cast<int>(input_length);
    const int nb = width / 256;
    for (uint32_t tok0 = 0; tok0 < batch;) {
        q38::StreamPlan plan;
        cudaError_t e = q38::stream_plan(static_cast<int>(tensor->type), rows, width,
                                         static_cast<int>(tensor->tile_rows), static_cast<int>(batch - tok0), &plan);
        if (e != cudaSuccess) return fail_cuda("stream plan", e);
        if (!tensor->scratch || tensor->scratch_bytes < plan.scratch_bytes)
            return fail("tensor scratch missing or too small (prepare it with q38cu_tensor_upload/repack)%s");
        const int tokens = plan.token_group;
        q38::StreamLaunch l;
        l.weights = tensor->data;
        l.act = input + static_cast<size_t>(tok0) * nb;
        l.tokens = tokens;
        l.out = output + static_cast<size_t>(tok0) * rows;
        l.scratch = tensor->scratch;
        l.dbg_w = w_out ? w_out + static_cast<size_t>(tok0) * rows * nb : nullptr;
        l.dbg_x = x_out ? x_out + static_cast<size_t>(tok0) * rows * nb : nullptr;
        e = q38::launch_stream_gemm(static_cast<int>(tensor->type), plan, l, stream);
        if (e != cudaSuccess) return fail_cuda("stream gemm launch", e);
        tok0 += static_cast<uint32_t>(tokens);
    }
    return 1;
}

// Scratch a tiled tensor needs for any batch size.
int stream_scratch_bytes(uint32_t type, uint64_t width, uint64_t rows, uint32_t tile_rows, uint64_t *bytes)
{
    uint64_t need = 0;
    for (int tokens = 1; tokens <= 8; ++tokens) {
        q38::StreamPlan plan;
        const cudaError_t e = q38::stream_plan(static_cast<int>(type), static_cast<int>(rows),
                                               static_cast<int>(width), static_cast<int>(tile_rows), tokens, &plan);
        if (e != cudaSuccess) return fail_cuda("stream plan", e);
        need = std::max(need, plan.scratch_bytes);
    }
    *bytes = need;
    return 1;
}

int gemm_q8k(float *output, int32_t *w_out, int32_t *x_out, const Q38CuQ8KBlock *input, uint32_t batch,
             uint64_t input_length, const Q38CuTensor *tensor, void *stream)
{
    if (!output || !input || !batch) return fail("output, input and batch_size are required%s");
    if (input_length % Q38CU_Q8_K_BLOCK_SIZE) return fail("input length must be a multiple of 256%s");
    if (!check_matrix(tensor, input_length)) return 0;
    if (!upstream_q8k_type(tensor->type)) return fail("type has no Q8_K integer kernel%s");
    if (!q38::superblock_bytes(static_cast<int>(tensor->type)))
        return fail("type not yet implemented on the device%s");
    if (input_length / 256 > 256) return fail("input length above 65536 is not supported%s");
    if (tensor->layout == Q38CU_LAYOUT_TILED)
        return stream_gemm(output, w_out, x_out, input, batch, input_length, tensor, static_cast<cudaStream_t>(stream));
    const q38::GemmPlan plan = make_plan(tensor->type, input_length, tensor->shape[1], static_cast<int>(batch));
    q38::LaunchGemm l{tensor->data, input, static_cast<int>(batch), output, w_out, x_out};
    const cudaError_t e =
        q38::launch_q8k_gemm(static_cast<int>(tensor->type), plan, l, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? 1 : fail_cuda("q8_k gemm launch", e);
}

}  // namespace

namespace q38 {

void set_last_error(const char *message) { std::snprintf(g_error, sizeof(g_error), "%s", message); }

int device_sm_count()
{
    static int counts[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!counts[dev]) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        counts[dev] = n > 0 ? n : 148;
    }
    return counts[dev];
}

}  // namespace q38

extern "C" {

float q38cu_f16_to_f32(uint16_t value)
{
    const uint32_t sign = static_cast<uint32_t>(value & 0x8000u) << 16;
    const uint32_t exponent = (value >> 10) & 31u;
    uint32_t mantissa = value & 1023u;
    uint32_t bits;
    if (exponent == 0) {
        if (mantissa == 0) {
            bits = sign;
        } else {
            int shifts = 0;
            while ((mantissa & 0x400u) == 0) { mantissa <<= 1; ++shifts; }
            bits = sign | static_cast<uint32_t>(113 - shifts) << 23 | (mantissa & 0x3ffu) << 13;
        }
    } else if (exponent == 31) {
        bits = sign | 0x7f800000u | mantissa << 13;
    } else {
        bits = sign | (exponent + 112u) << 23 | mantissa << 13;
    }
    float out;
    std::memcpy(&out, &bits, sizeof(out));
    return out;
}

uint32_t q38cu_block_bytes(uint32_t type) { return geometry(type).bytes; }
uint32_t q38cu_block_elements(uint32_t type) { return geometry(type).elements; }

const char *q38cu_last_error(void) { return g_error; }

int q38cu_device_status(void *stream)
{
    int status = 0, stream_status = 0, tc_status = 0;
    cudaError_t e = q38::read_and_clear_status(&status, static_cast<cudaStream_t>(stream));
    if (e == cudaSuccess) e = q38::read_and_clear_stream_status(&stream_status);
    if (e == cudaSuccess) e = q38::read_and_clear_tc_status(&tc_status);
    if (e != cudaSuccess) {
        fail_cuda("device status", e);
        return -1;
    }
    return status ? status : stream_status ? stream_status : tc_status;
}

uint64_t q38cu_gguf_check(const char *path)
{
    if (!path) return fail("path is required%s");
    q38::GGUFFile f;
    if (!f.open(path)) return fail("%s", f.error().c_str());
    return f.tensor_count();
}

int q38cu_debug_wait_probe(uint64_t limit_ns, void *stream)
{
    if (limit_ns == 0 || limit_ns > 1000000000ull) return fail("limit_ns must be in 1 .. 1e9%s");
    const cudaError_t e = q38::launch_wait_probe(limit_ns, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? 1 : fail_cuda("wait probe launch", e);
}

int q38cu_quantize_q8_k(Q38CuQ8KBlock *output, const float *input, uint64_t length, void *stream)
{
    if (!output || !input) return fail("output and input are required%s");
    if (length % Q38CU_Q8_K_BLOCK_SIZE) return fail("length must be a multiple of 256%s");
    if (reinterpret_cast<uintptr_t>(input) & 15u) return fail("input must be 16-byte aligned%s");
    if (reinterpret_cast<uintptr_t>(output) & 3u) return fail("output must be 4-byte aligned%s");
    const cudaError_t e = q38::launch_quantize_q8k(output, input, length / 256, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? 1 : fail_cuda("quantize launch", e);
}

int q38cu_tensor_gemv_q8_k(float *output, const Q38CuQ8KBlock *input, uint64_t input_length,
                           const Q38CuTensor *tensor, void *stream)
{
    return gemm_q8k(output, nullptr, nullptr, input, 1, input_length, tensor, stream);
}

int q38cu_tensor_gemm_q8_k(float *output, const Q38CuQ8KBlock *input, uint32_t batch_size,
                           uint64_t input_length, const Q38CuTensor *tensor, void *stream)
{
    return gemm_q8k(output, nullptr, nullptr, input, batch_size, input_length, tensor, stream);
}

namespace {
// Workspace of q38cu_tensor_gemm_q8_k_tc: A hi/lo fp16 [2][rows][K], B fp16
// [batch][K], block scales [K / 256][ld], row powers of two [rows]; each
// part 256-byte aligned.
struct TcWorkspace {
    uint64_t a, b, scale, row_scale, total;
    uint32_t ld;
};
TcWorkspace tc_workspace_layout(uint64_t batch, uint64_t width, uint64_t rows)
{
    auto up = [](uint64_t x) { return (x + 255) / 256 * 256; };
    TcWorkspace w;
    const uint64_t tile = static_cast<uint64_t>(q38::tc_token_tile(static_cast<int>(batch)));
    w.ld = static_cast<uint32_t>((batch + tile - 1) / tile * tile);
    w.a = 0;
    w.b = up(rows * width * 4);
    w.scale = w.b + up(batch * width * 2);
    w.row_scale = w.scale + up(width / 256 * w.ld * 4);
    w.total = w.row_scale + up(rows * 4);
    return w;
}
}  // namespace

uint64_t q38cu_tensor_gemm_q8_k_tc_workspace(uint32_t batch_size, uint64_t input_length, const Q38CuTensor *tensor)
{
    if (!tensor || !batch_size || tensor->n_dims != 2 || input_length % 256) return 0;
    return tc_workspace_layout(batch_size, input_length, tensor->shape[1]).total;
}

int q38cu_tensor_gemm_q8_k_tc(float *output, const Q38CuQ8KBlock *input, uint32_t batch_size, uint64_t input_length,
                              const Q38CuTensor *tensor, void *workspace, uint64_t workspace_bytes, void *stream)
{
    if (!output || !input || !batch_size || !workspace) return fail("output, input, batch_size and workspace are required%s");
    if (!check_matrix(tensor, input_length)) return 0;
    if (!q38::tc_weight_type(static_cast<int>(tensor->type)))
        return fail("the tensor-core GEMM takes Q4_K and Q6_K weights%s");
    if (input_length % 256 || input_length > (1u << 20) || batch_size > (1u << 20))
        return fail("input length must be a multiple of 256; batch and width at most 2^20%s");
    if (!aligned16(output) || !aligned16(input)) return fail("output and input must be 16-byte aligned%s");
    if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return fail("workspace must be 256-byte aligned%s");
    const uint64_t need = q38cu_tensor_gemm_q8_k_tc_workspace(batch_size, input_length, tensor);
    if (workspace_bytes < need) return fail("workspace smaller than q38cu_tensor_gemm_q8_k_tc_workspace()%s");
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    const TcWorkspace lay = tc_workspace_layout(batch_size, input_length, tensor->shape[1]);
    void *a16 = ws + lay.a;
    void *b16 = ws + lay.b;
    float *scale = reinterpret_cast<float *>(ws + lay.scale);
    float *row_scale = reinterpret_cast<float *>(ws + lay.row_scale);
    const Geometry g = geometry(tensor->type);
    cudaError_t e = q38::launch_dequant_f16(tensor->data, static_cast<int>(tensor->type), tensor->shape[1],
                                            input_length, layout_tile_rows(tensor), static_cast<int>(g.bytes), a16,
                                            row_scale, 0, s);
    if (e == cudaSuccess)
        e = q38::launch_q8k_to_f16(input, static_cast<int>(input_length / 256), static_cast<int>(batch_size),
                                   static_cast<int>(lay.ld), b16, scale, s);
    if (e == cudaSuccess) {
        q38::TcGemm p;
        p.out = output;
        p.ld = static_cast<int>(tensor->shape[1]);
        p.n = static_cast<int>(tensor->shape[1]);
        p.m = static_cast<int>(batch_size);
        p.k = static_cast<int>(input_length);
        p.b_scale = scale;
        p.b_scale_ld = static_cast<int>(lay.ld);
        p.row_scale = row_scale;
        p.accumulate = 0;
        e = q38::launch_tc_gemm(a16, b16, p, s);
    }
    return e == cudaSuccess ? 1 : fail_cuda("tensor-core gemm launch", e);
}

int q38cu_tensor_gemm_q8_k_sums(float *output, int32_t *w_out, int32_t *x_out, const Q38CuQ8KBlock *input,
                                uint32_t batch_size, uint64_t input_length, const Q38CuTensor *tensor,
                                void *stream)
{
    if (!w_out || !x_out) return fail("sum outputs are required%s");
    // IQ4_NL accumulates floats per 32-element block: no integer superblock sums.
    if (tensor && tensor->type == 20) return fail("IQ4_NL has no integer superblock sums%s");
    return gemm_q8k(output, w_out, x_out, input, batch_size, input_length, tensor, stream);
}

int q38cu_tensor_gemm_f32(float *output, const float *input, uint32_t batch_size, uint64_t input_length,
                          const Q38CuTensor *tensor, void *stream)
{
    if (!output || !input || !batch_size) return fail("output, input and batch_size are required%s");
    if (!check_matrix(tensor, input_length)) return 0;
    if (!float_path_type(tensor->type)) return fail("type has no float-path kernel%s");
    const Geometry g = geometry(tensor->type);
    const cudaError_t e = q38::launch_f32_gemm(output, input, static_cast<int>(batch_size), input_length,
                                               tensor->data, tensor->shape[1], layout_tile_rows(tensor),
                                               static_cast<int>(tensor->type),
                                               static_cast<int>(g.elements), static_cast<int>(g.bytes),
                                               static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? 1 : fail_cuda("f32 gemm launch", e);
}

int q38cu_tensor_gemv_f32(float *output, const float *input, const Q38CuTensor *tensor, void *stream)
{
    if (!tensor) return fail("tensor is NULL%s");
    return q38cu_tensor_gemm_f32(output, input, 1, tensor->shape[0], tensor, stream);
}

int q38cu_tensor_row_f32(float *output, const Q38CuTensor *tensor, uint64_t row, void *stream)
{
    if (!output || !tensor) return fail("output and tensor are required%s");
    if (!check_matrix(tensor, tensor->shape[0])) return 0;
    if (row >= tensor->shape[1]) return fail("row out of range%s");
    if (!float_path_type(tensor->type)) return fail("type has no row decoder%s");
    const Geometry g = geometry(tensor->type);
    const cudaError_t e = q38::launch_row_f32(output, tensor->data, tensor->shape[0], layout_tile_rows(tensor), row,
                                              static_cast<int>(tensor->type), static_cast<int>(g.elements),
                                              static_cast<int>(g.bytes), static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? 1 : fail_cuda("row launch", e);
}

int q38cu_tensor_dot_row_f32(float *output, const float *input, const Q38CuTensor *tensor, uint64_t row,
                             void *stream)
{
    if (!output || !input || !tensor) return fail("output, input and tensor are required%s");
    if (!check_matrix(tensor, tensor->shape[0])) return 0;
    if (row >= tensor->shape[1]) return fail("row out of range%s");
    if (!float_path_type(tensor->type)) return fail("type has no float-path kernel%s");
    const Geometry g = geometry(tensor->type);
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = q38::launch_dot_row_f32(output, input, tensor->data, tensor->shape[0], layout_tile_rows(tensor),
                                            row, static_cast<int>(tensor->type), static_cast<int>(g.elements),
                                            static_cast<int>(g.bytes), s);
    float host = 0.0f;
    if (e == cudaSuccess) e = cudaMemcpyAsync(&host, output, sizeof(float), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return fail_cuda("dot row", e);
    return std::isfinite(host) ? 1 : fail("the row's dot product is not finite%s");
}

int q38cu_tensor_upload(Q38CuTensor *tensor, uint32_t type, uint64_t width, uint64_t rows, const void *host_data,
                        uint32_t layout, void *stream)
{
    if (!tensor) return fail("tensor is NULL%s");
    const Geometry g = geometry(type);
    if (!g.elements || !width || width % g.elements || !rows) return fail("unsupported type or shape%s");
    if (layout != Q38CU_LAYOUT_GGUF && layout != Q38CU_LAYOUT_TILED) return fail("unknown layout%s");
    if (layout == Q38CU_LAYOUT_TILED && !superblock_layout_type(type))
        return fail("tiled layout needs a 256-element block type%s");
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    Q38CuTensor src{};
    src.type = type;
    src.n_dims = 2;
    src.shape[0] = width;
    src.shape[1] = rows;
    src.nbytes = width / g.elements * g.bytes * rows;
    src.layout = Q38CU_LAYOUT_GGUF;
    void *dev = nullptr;
    cudaError_t e = cudaMalloc(&dev, (src.nbytes + 15) / 16 * 16 + 256);
    if (e != cudaSuccess) return fail_cuda("cudaMalloc", e);
    if (host_data) {
        e = cudaMemcpyAsync(dev, host_data, src.nbytes, cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) {
            cudaFree(dev);
            return fail_cuda("upload copy", e);
        }
    }
    src.data = dev;
    if (layout == Q38CU_LAYOUT_GGUF) {
        *tensor = src;
        return 1;
    }
    const int ok = q38cu_tensor_repack(tensor, &src, stream);
    cudaStreamSynchronize(s);
    cudaFree(dev);
    return ok;
}

int q38cu_tensor_repack(Q38CuTensor *dst, const Q38CuTensor *src, void *stream)
{
    return q38::repack_tiled_with(dst, src, 0, stream);
}

}  // extern "C"

namespace q38 {

// q38cu_tensor_repack with a caller-chosen tile height (0: the default for the
// row count).
int repack_tiled_with(void *dst_tensor, const void *src_tensor, uint32_t forced_tile_rows, void *stream)
{
    Q38CuTensor *dst = static_cast<Q38CuTensor *>(dst_tensor);
    const Q38CuTensor *src = static_cast<const Q38CuTensor *>(src_tensor);
    if (!dst || !src) return fail("dst and src are required%s");
    if (!check_matrix(src, src->shape[0])) return 0;
    if (src->layout != Q38CU_LAYOUT_GGUF) return fail("source must be in the GGUF layout%s");
    if (!superblock_layout_type(src->type)) return fail("tiled layout needs a 256-element block type%s");
    if (!q38::superblock_bytes(static_cast<int>(src->type))) return fail("type not yet implemented on the device%s");
    const Geometry g = geometry(src->type);
    const uint64_t nb = src->shape[0] / 256, rows = src->shape[1];
    if (forced_tile_rows && (forced_tile_rows % 8 || forced_tile_rows > 256)) return fail("bad tile height%s");
    const uint32_t tile_rows =
        forced_tile_rows ? forced_tile_rows : static_cast<uint32_t>(q38::stream_tile_rows(static_cast<int>(rows)));
    const uint64_t nbytes = nb * g.bytes * rows_padded(rows, tile_rows);
    uint64_t scratch_bytes = 0;
    if (!stream_scratch_bytes(src->type, src->shape[0], rows, tile_rows, &scratch_bytes)) return 0;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    void *data = nullptr, *scratch = nullptr;
    cudaError_t e = cudaMalloc(&data, nbytes + 256);
    if (e == cudaSuccess) e = cudaMalloc(&scratch, scratch_bytes);
    if (e == cudaSuccess) e = cudaMemsetAsync(data, 0, nbytes + 256, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(scratch, 0, scratch_bytes, s);
    if (e == cudaSuccess) e = q38::launch_repack_tiled(data, src->data, rows, nb, tile_rows, g.bytes, s);
    if (e != cudaSuccess) {
        cudaFree(data);
        cudaFree(scratch);
        return fail_cuda("repack", e);
    }
    Q38CuTensor t{};
    t.type = src->type;
    t.n_dims = 2;
    t.shape[0] = src->shape[0];
    t.shape[1] = rows;
    t.nbytes = nbytes;
    t.data = data;
    t.layout = Q38CU_LAYOUT_TILED;
    t.tile_rows = tile_rows;
    t.scratch = scratch;
    t.scratch_bytes = scratch_bytes;
    *dst = t;
    return 1;
}

}  // namespace q38

extern "C" {

void q38cu_tensor_free(Q38CuTensor *tensor)
{
    if (!tensor) return;
    if (tensor->data) cudaFree(const_cast<void *>(tensor->data));
    if (tensor->scratch) cudaFree(tensor->scratch);
    tensor->data = nullptr;
    tensor->scratch = nullptr;
    tensor->scratch_bytes = 0;
}

}  // extern "C"
