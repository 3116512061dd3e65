// Allocation-free sampling entry point (rsc_sample_noalloc).
//
// Who needs it: a host program that hands the library only raw device
// pointers and cannot let it allocate. Examples are an inference server that
// reserves nearly all of HBM for its KV cache at start-up and fails any later
// cudaMalloc; a runtime that owns device memory through its own pool and
// forbids a library from growing outside it; and a plugin that has no
// lifetime hook in which a handle's memory could be freed. Such callers
// cannot use rsc_sampler_create, which allocates the handle's scratch.
//
// How: the large-survivor kernel (sample_large.cu) runs on every row, with
// its sorting scratch taken from kNoAllocScratch below, a fixed array in the
// library's own device image. Its address is looked up once per device with
// cudaGetSymbolAddress; nothing here calls cudaMalloc, cudaFree or any
// allocating routine. The scratch needs no clearing: the kernel writes every
// word of it before reading it.
//
// Limits: the array holds RSC_NOALLOC_SCRATCH_BYTES; a call needs
// 16 * vocab bytes per concurrently sampled row, so vocab is at most
// RSC_NOALLOC_SCRATCH_BYTES / 16 and larger vocabularies are rejected with
// RSC_ERR_CAPACITY; vocab 0 with rows > 0 is RSC_ERR_INVALID_SHAPE. Every
// call on a device shares the one array, so calls whose kernels overlap on
// the GPU (different streams, no ordering between them) race on it; order
// them on one stream or with events.
#include <cuda_runtime.h>

#include <cmath>
#include <mutex>

#include "rsc_kernels.h"

namespace {

constexpr size_t kScratchWords = RSC_NOALLOC_SCRATCH_BYTES / sizeof(uint32_t);
constexpr size_t kMaxDevices = 64;

// The scratch: one per device that loads the library, kept until exit.
static __device__ __align__(256) uint32_t kNoAllocScratch[kScratchWords];

struct DeviceSetup {
    std::mutex mu;
    bool ready = false;           // set only by a set-up that succeeded
    uint32_t *scratch = nullptr;  // device address of kNoAllocScratch
    int num_sms = 0;
};

DeviceSetup g_setup[kMaxDevices];

// Set-up of `device`, which must be current: the device address of the
// scratch array (a host-side reference to the symbol is not a device
// address) and the SM count. Only a successful set-up is kept; after a
// failure (for example a first call made inside a stream capture) the next
// call tries again.
cudaError_t setup_device(int device, DeviceSetup **out) {
    DeviceSetup *s = &g_setup[device];
    std::lock_guard<std::mutex> lock(s->mu);
    if (!s->ready) {
        void *ptr = nullptr;
        int sms = 0;
        cudaError_t e = cudaGetSymbolAddress(&ptr, kNoAllocScratch);
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
        if (e != cudaSuccess || !ptr || sms <= 0) return e != cudaSuccess ? e : cudaErrorUnknown;
        s->scratch = static_cast<uint32_t *>(ptr);
        s->num_sms = sms;
        s->ready = true;
    }
    *out = s;
    return cudaSuccess;
}

}  // namespace

extern "C" RSC_API rsc_status rsc_sample_noalloc(const float *d_logits, size_t rows, size_t vocab,
                                                 size_t row_stride, const rsc_params *params,
                                                 const float *d_uniforms, uint64_t *d_rng_states,
                                                 uint32_t *d_out_ids, int32_t *d_out_status,
                                                 float *d_out_probs, void *stream) {
    if (!params) return RSC_ERR_INVALID_ARGUMENT;
    if (vocab >= (size_t{1} << 31)) return RSC_ERR_VOCAB_TOO_LARGE;
    if (vocab > RSC_NOALLOC_MAX_VOCAB) return RSC_ERR_CAPACITY;
    if (rows > 0 && vocab > 0 && row_stride < vocab) return RSC_ERR_INVALID_SHAPE;
    if (rows == 0) return RSC_OK;
    if (vocab == 0) return RSC_ERR_INVALID_SHAPE;
    if (!d_out_ids || !d_out_status || (vocab > 0 && !d_logits)) return RSC_ERR_INVALID_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(d_logits) & 3u) != 0) return RSC_ERR_INVALID_ARGUMENT;
    const bool argmax = params->temperature == 0.0f || params->top_k == 1;
    if (!argmax && !d_uniforms && !d_rng_states) return RSC_ERR_INVALID_ARGUMENT;

    int device = -1;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0) return RSC_ERR_NO_DEVICE;
    if (static_cast<size_t>(device) >= kMaxDevices) return RSC_ERR_NO_DEVICE;
    DeviceSetup *s = nullptr;
    if (setup_device(device, &s) != cudaSuccess) return RSC_ERR_CUDA;

    rsc::CallParams cp;
    cp.temperature = params->temperature;
    cp.scale = params->temperature > 0.0f ? 1.0f / params->temperature : 1.0f;
    cp.top_k = params->top_k;
    cp.top_p = params->top_p;
    cp.topk_active = params->top_k != 0 && static_cast<size_t>(params->top_k) < vocab;
    cp.topp_active = params->top_p < 1.0f;
    cp.argmax_branch = argmax;
    // As rsc_sample derives it: it sends rows with no filter at a normal scale
    // to the large kernel's filter-free branch, with the same results.
    cp.normal_scale = std::isfinite(cp.scale) && cp.scale > 0.0f;
    cp.mode = rsc::kModeSampleLogits;
    cp.uniforms = d_uniforms;
    cp.rng_states = d_rng_states;
    cp.out_nsurv = nullptr;
    cp.out_surv = nullptr;
    cp.surv_cap = 0;

    // Rows sampled at once: kLargeCtasPerSm per SM, as many as the scratch holds.
    const size_t per_row = 4 * vocab;
    size_t slots = kScratchWords / per_row;
    const size_t resident = static_cast<size_t>(s->num_sms) * rsc::kLargeCtasPerSm;
    if (slots > resident) slots = resident;
    if (slots > rows) slots = rows;
    cudaError_t e = rsc::launch_large(d_logits, rows, static_cast<uint32_t>(vocab), row_stride, cp,
                                      d_out_ids, d_out_status, d_out_probs,
                                      s->scratch, static_cast<uint32_t>(slots),
                                      static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? RSC_OK : RSC_ERR_CUDA;
}
