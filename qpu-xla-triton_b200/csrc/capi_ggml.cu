// GGML MUL_MAT offload core (include/qpucuda_ggml.h): the node-level work of the reference's
// llama.cpp backend (integrations/llama_cpp/backend/ggml-qpu.cpp:245-377, 539-620) over a plain
// tensor view, on top of the prepared Q4_0 linear of capi_q4_0.cu.
#include <chrono>
#include <cstring>
#include <mutex>
#include <new>
#include <unordered_map>
#include <vector>

#include "qpucuda_ggml.h"
#include "qpucuda_internal.h"
#include "qpucuda_q4_0.h"

using namespace qpucuda;

namespace {

constexpr size_t kQ40BlockBytes = 18;  // fp16 d + 16 nibble bytes
constexpr uint32_t kMaxRows = 4u * 65535u;

struct CachedLinear {
    qpucuda_q4_0_linear *linear = nullptr;
    uint32_t row_capacity = 0;
    // What the plan was prepared from: a key reused by a different tensor (freed and
    // reallocated at the same address) does not match and is prepared afresh.
    const void *data = nullptr;
    int64_t input_columns = 0;
    int64_t output_columns = 0;
    int32_t cpu_repack = 0;
};

bool contiguous_f32(const qpucuda_ggml_tensor *t) {
    return t->nb[0] == sizeof(float) && t->nb[1] == t->nb[0] * static_cast<size_t>(t->ne[0]) &&
           t->nb[2] == t->nb[1] * static_cast<size_t>(t->ne[1]) && t->nb[3] == t->nb[2] * static_cast<size_t>(t->ne[2]);
}

// Q4_0 blocks packed row after row ([N][K/32][18 bytes]): the only weight layout the prepare
// copies from.
bool contiguous_q4_0(const qpucuda_ggml_tensor *t) {
    return t->nb[0] == kQ40BlockBytes && t->nb[1] == kQ40BlockBytes * static_cast<size_t>(t->ne[0] / 32) &&
           t->nb[2] == t->nb[1] * static_cast<size_t>(t->ne[1]) && t->nb[3] == t->nb[2] * static_cast<size_t>(t->ne[2]);
}

uint64_t now_ns() {
    return static_cast<uint64_t>(
        std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now().time_since_epoch())
            .count());
}

}  // namespace

struct qpucuda_ggml_backend {
    qpucuda_context *context = nullptr;
    uint32_t minimum_rows = 1;
    uint32_t maximum_rows = kMaxRows;
    std::mutex mutex;  // one node at a time, like the reference's graph_compute lock
    std::unordered_map<const void *, CachedLinear> linears;
    float *d_source = nullptr;  // F32 activation rows on the device
    size_t source_floats = 0;
    float *d_output = nullptr;  // fp32 result on the device
    size_t output_floats = 0;
    float *h_output = nullptr;  // pinned staging of the result
    size_t host_floats = 0;
    qpucuda_ggml_stats stats{};
};

namespace {

void release_staging(qpucuda_ggml_backend *backend) {
    cudaFree(backend->d_source);
    cudaFree(backend->d_output);
    cudaFreeHost(backend->h_output);
    (void)cudaGetLastError();
    backend->d_source = backend->d_output = backend->h_output = nullptr;
    backend->source_floats = backend->output_floats = backend->host_floats = 0;
}

// Grows the staging to hold `source` input and `output` result floats (allocations happen only
// when a call needs more than any earlier one).
qpucuda_status ensure_staging(qpucuda_ggml_backend *backend, size_t source, size_t output) {
    qpucuda_context *context = backend->context;
    if (source <= backend->source_floats && output <= backend->output_floats && output <= backend->host_floats) {
        return QPUCUDA_OK;
    }
    release_staging(backend);
    if ((context->failure_mask & QPUCUDA_FAIL_ALLOCATION) != 0 ||
        cudaMalloc(reinterpret_cast<void **>(&backend->d_source), source * sizeof(float)) != cudaSuccess ||
        cudaMalloc(reinterpret_cast<void **>(&backend->d_output), output * sizeof(float)) != cudaSuccess ||
        cudaMallocHost(reinterpret_cast<void **>(&backend->h_output), output * sizeof(float)) != cudaSuccess) {
        release_staging(backend);
        return fail(context, QPUCUDA_ALLOCATION_FAILED, "GGML offload: allocate staging");
    }
    backend->source_floats = source;
    backend->output_floats = output;
    backend->host_floats = output;
    return QPUCUDA_OK;
}

// get_or_prepare_linear (ggml-qpu.cpp:319-360): a cached plan serves any call with at most its
// row capacity on the same weight (data pointer, shape, layout); otherwise it is replaced.
qpucuda_status get_or_prepare(qpucuda_ggml_backend *backend, const qpucuda_ggml_tensor *weight, uint32_t rows,
                              qpucuda_q4_0_linear **result) {
    const void *key = weight->identity != nullptr ? weight->identity : weight->data;
    auto existing = backend->linears.find(key);
    if (existing != backend->linears.end() && existing->second.row_capacity >= rows &&
        existing->second.data == weight->data && existing->second.input_columns == weight->ne[0] &&
        existing->second.output_columns == weight->ne[1] && existing->second.cpu_repack == weight->cpu_repack) {
        ++backend->stats.weight_cache_hits;
        *result = existing->second.linear;
        return QPUCUDA_OK;
    }
    if (existing != backend->linears.end()) {
        qpucuda_q4_0_linear_destroy(existing->second.linear);
        backend->linears.erase(existing);
    }
    const uint32_t k = static_cast<uint32_t>(weight->ne[0]);
    const uint32_t n = static_cast<uint32_t>(weight->ne[1]);
    const size_t native_size = static_cast<size_t>(n) * (k / 32) * kQ40BlockBytes;
    std::vector<uint8_t> unpacked;
    const void *native = weight->data;
    if (weight->cpu_repack != 0) {
        try {
            unpacked.resize(native_size);
        } catch (const std::bad_alloc &) {
            return fail(backend->context, QPUCUDA_ALLOCATION_FAILED, "GGML offload: unpack buffer");
        }
        const qpucuda_status status =
            qpucuda_ggml_unpack_q4_0x4(weight->data, native_size, k, n, unpacked.data(), unpacked.size());
        if (status != QPUCUDA_OK) return status;
        native = unpacked.data();
    }
    qpucuda_q4_0_linear_desc desc{};
    desc.weights = native;
    desc.weight_size = native_size;
    desc.input_columns = k;
    desc.output_columns = n;
    desc.rows = rows;
    desc.resident_column_start = 0;
    desc.resident_column_count = n;
    desc.weight_mode = QPUCUDA_Q4_0_WEIGHT_EXACT;
    desc.workgroups_per_supergroup = 24;
    desc.expected_source_hash = qpucuda_q4_0_kernel_source_hash();
    qpucuda_q4_0_linear *prepared = nullptr;
    const qpucuda_status status = qpucuda_q4_0_linear_prepare(backend->context, &desc, &prepared);
    if (status != QPUCUDA_OK) return status;
    try {
        backend->linears.emplace(key, CachedLinear{prepared, rows, weight->data, weight->ne[0], weight->ne[1],
                                                   weight->cpu_repack});
    } catch (...) {
        qpucuda_q4_0_linear_destroy(prepared);  // no exception crosses the C ABI
        return fail(backend->context, QPUCUDA_ALLOCATION_FAILED, "GGML offload: weight cache entry");
    }
    ++backend->stats.weight_cache_misses;
    *result = prepared;
    return QPUCUDA_OK;
}

}  // namespace

extern "C" {

int qpucuda_ggml_supports_mul_mat(const qpucuda_ggml_tensor *weight, const qpucuda_ggml_tensor *activation,
                                  const qpucuda_ggml_tensor *destination, uint32_t minimum_rows,
                                  uint32_t maximum_rows) {
    if (weight == nullptr || activation == nullptr || destination == nullptr || weight->data == nullptr ||
        activation->data == nullptr || destination->data == nullptr) {
        return 0;
    }
    // supports_q4_0_mul_mat (ggml-qpu.cpp:362-377)
    const bool shape = weight->type == QPUCUDA_GGML_TYPE_Q4_0 && activation->type == QPUCUDA_GGML_TYPE_F32 &&
                       weight->ne[0] > 0 && weight->ne[0] % 32 == 0 && weight->ne[1] > 0 && weight->ne[1] % 16 == 0 &&
                       activation->ne[0] == weight->ne[0] && activation->ne[1] > 0 &&
                       activation->ne[1] <= static_cast<int64_t>(kMaxRows) && weight->ne[2] == 1 &&
                       weight->ne[3] == 1 && activation->ne[2] == 1 && activation->ne[3] == 1 &&
                       contiguous_f32(activation);
    // the MUL_MAT node's own tensor: F32 [N, M], contiguous
    const bool result = destination->type == QPUCUDA_GGML_TYPE_F32 && destination->ne[0] == weight->ne[1] &&
                        destination->ne[1] == activation->ne[1] && destination->ne[2] == 1 &&
                        destination->ne[3] == 1 && contiguous_f32(destination);
    // unpack_q4_0_4x4 needs whole 4-row groups (ggml-qpu.cpp:257-261). The weight must also be
    // contiguous, which the reference assumes without checking: a strided view falls back to
    // another backend here instead of being read as packed blocks.
    const bool layout = (weight->cpu_repack == 0 || weight->ne[1] % 4 == 0) && contiguous_q4_0(weight);
    // the device's row window (ggml-qpu.cpp:631-633)
    const bool window = activation->ne[1] >= static_cast<int64_t>(minimum_rows) &&
                        activation->ne[1] <= static_cast<int64_t>(maximum_rows);
    return shape && result && layout && window ? 1 : 0;
}

qpucuda_status qpucuda_ggml_unpack_q4_0x4(const void *packed, size_t packed_size, uint32_t input_columns,
                                          uint32_t output_columns, void *native, size_t native_size) {
    if (packed == nullptr || native == nullptr || input_columns == 0 || input_columns % 32 != 0 ||
        output_columns == 0 || output_columns % 4 != 0) {
        return QPUCUDA_INVALID_ARGUMENT;
    }
    const size_t blocks = input_columns / 32;
    const size_t bytes = static_cast<size_t>(output_columns) * blocks * kQ40BlockBytes;
    if (packed_size < bytes || native_size < bytes) return QPUCUDA_INVALID_ARGUMENT;
    const uint8_t *source = static_cast<const uint8_t *>(packed);
    uint8_t *out = static_cast<uint8_t *>(native);
    // One group holds 4 weight rows; per K block: their 4 scales (8 bytes), then 64 quant bytes in
    // which 4-byte chunk c of row r sits at (c * 4 + r) * 4, every byte XOR 0x88.
    for (size_t group = 0; group < output_columns / 4u; ++group) {
        for (size_t block = 0; block < blocks; ++block) {
            const uint8_t *in = source + (group * blocks + block) * 4 * kQ40BlockBytes;
            for (size_t row = 0; row < 4; ++row) {
                uint8_t *dst = out + ((group * 4 + row) * blocks + block) * kQ40BlockBytes;
                dst[0] = in[row * 2];
                dst[1] = in[row * 2 + 1];
                for (size_t chunk = 0; chunk < 4; ++chunk) {
                    const uint8_t *quads = in + 8 + (chunk * 4 + row) * 4;
                    for (size_t byte = 0; byte < 4; ++byte) dst[2 + chunk * 4 + byte] = quads[byte] ^ 0x88u;
                }
            }
        }
    }
    return QPUCUDA_OK;
}

qpucuda_status qpucuda_ggml_backend_create(qpucuda_context *context, uint32_t minimum_rows, uint32_t maximum_rows,
                                           qpucuda_ggml_backend **result) {
    if (result == nullptr) return QPUCUDA_INVALID_ARGUMENT;
    *result = nullptr;
    if (context == nullptr || minimum_rows == 0 || minimum_rows > maximum_rows) return QPUCUDA_INVALID_ARGUMENT;
    qpucuda_ggml_backend *backend = new (std::nothrow) qpucuda_ggml_backend();
    if (backend == nullptr) return fail(context, QPUCUDA_ALLOCATION_FAILED, "GGML offload: backend");
    backend->context = context;
    backend->minimum_rows = minimum_rows;
    backend->maximum_rows = maximum_rows < kMaxRows ? maximum_rows : kMaxRows;
    *result = backend;
    return QPUCUDA_OK;
}

void qpucuda_ggml_backend_destroy(qpucuda_ggml_backend *backend) {
    if (backend == nullptr) return;
    {
        std::lock_guard<std::mutex> lock(backend->mutex);
        for (auto &entry : backend->linears) qpucuda_q4_0_linear_destroy(entry.second.linear);
        backend->linears.clear();
        DeviceGuard guard(backend->context->device);
        release_staging(backend);
    }
    delete backend;
}

void qpucuda_ggml_backend_forget(qpucuda_ggml_backend *backend, const void *identity) {
    if (backend == nullptr) return;
    std::lock_guard<std::mutex> lock(backend->mutex);
    auto existing = backend->linears.find(identity);
    if (existing == backend->linears.end()) return;
    qpucuda_q4_0_linear_destroy(existing->second.linear);
    backend->linears.erase(existing);
}

qpucuda_status qpucuda_ggml_backend_stats(const qpucuda_ggml_backend *backend, qpucuda_ggml_stats *result) {
    if (backend == nullptr || result == nullptr) return QPUCUDA_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> lock(const_cast<qpucuda_ggml_backend *>(backend)->mutex);
    *result = backend->stats;
    return QPUCUDA_OK;
}

qpucuda_status qpucuda_ggml_mul_mat(qpucuda_ggml_backend *backend, const qpucuda_ggml_tensor *weight,
                                    const qpucuda_ggml_tensor *activation, qpucuda_ggml_tensor *destination) {
    if (backend == nullptr) return QPUCUDA_INVALID_ARGUMENT;
    qpucuda_context *context = backend->context;
    if (!qpucuda_ggml_supports_mul_mat(weight, activation, destination, backend->minimum_rows,
                                       backend->maximum_rows)) {
        return fail(context, QPUCUDA_INVALID_ARGUMENT, "GGML offload: unsupported MUL_MAT node");
    }
    std::lock_guard<std::mutex> lock(backend->mutex);
    const uint64_t start = now_ns();
    const uint32_t k = static_cast<uint32_t>(weight->ne[0]);
    const uint32_t n = static_cast<uint32_t>(weight->ne[1]);
    const uint32_t rows = static_cast<uint32_t>(activation->ne[1]);
    DeviceGuard guard(context->device);
    qpucuda_q4_0_linear *linear = nullptr;
    qpucuda_status status = get_or_prepare(backend, weight, rows, &linear);
    if (status != QPUCUDA_OK) return status;
    status = ensure_staging(backend, static_cast<size_t>(rows) * k, static_cast<size_t>(rows) * n);
    if (status != QPUCUDA_OK) return status;
    const size_t source_bytes = static_cast<size_t>(rows) * k * sizeof(float);
    const size_t output_bytes = static_cast<size_t>(rows) * n * sizeof(float);
    {
        std::lock_guard<std::mutex> context_lock(context->mutex);
        status = begin_submit(context);
        if (status != QPUCUDA_OK) return status;
        const cudaError_t error =
            cudaMemcpyAsync(backend->d_source, activation->data, source_bytes, cudaMemcpyHostToDevice, context->stream);
        if (error != cudaSuccess) return cuda_fail(context, error, "GGML offload: copy activation rows");
    }
    const uint64_t copied = now_ns();
    // Q8_0 quantization of the F32 rows happens inside the kernel (matvec for rows <= 4, the
    // tensor-core tiled path above), bit-identical to quantize_row_q8_0 then the Q8_0 kernel.
    status = qpucuda_q4_0_linear_execute_f32_device(linear, backend->d_source, k, rows, backend->d_output, n, 0, n, 0);
    if (status != QPUCUDA_OK) return status;
    {
        std::lock_guard<std::mutex> context_lock(context->mutex);
        const cudaError_t error =
            cudaMemcpyAsync(backend->h_output, backend->d_output, output_bytes, cudaMemcpyDeviceToHost, context->stream);
        if (error != cudaSuccess) return cuda_fail(context, error, "GGML offload: copy result");
        status = wait_stream(context);  // bounded; a failure poisons the context
    }
    const uint64_t waited = now_ns();
    if (status != QPUCUDA_OK) return status;  // destination untouched
    parallel_memcpy(destination->data, backend->h_output, output_bytes);
    const uint64_t end = now_ns();
    ++backend->stats.dispatch_count;
    backend->stats.input_copy_ns = copied - start;
    backend->stats.submit_wait_ns = waited - copied;
    backend->stats.output_copy_ns = end - waited;
    backend->stats.complete_ns = end - start;
    backend->stats.rows = rows;
    return QPUCUDA_OK;
}

}  // extern "C"
