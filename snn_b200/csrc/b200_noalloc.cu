// snn_b200_step_noalloc: one push-mode simulation step over caller-owned
// device arrays that allocates no memory at all.
//
// Why it exists: some callers cannot call cudaMalloc (or anything that
// allocates) once they are running -- code whose device memory is entirely
// owned by an outer framework's pool or arena, real-time or safety-critical
// loops where allocation after start-up is forbidden, and launchers that must
// not trigger the implicit synchronisation an allocation can cause. Such a
// caller allocates the network and state arrays itself, once, and this entry
// point works only inside them plus a fixed scratch area compiled into the
// library.
//
// The scratch area (spike list, spike bitmap, step counters) is a file-scope
// __device__ array of fixed size. Every GPU that loads the library holds it
// until the process exits, and every call on a device shares the one copy:
// calls whose work overlaps on the GPU (for example on two streams at once)
// race on it and must be serialised by the caller. The array keeps whatever
// the last call left in it; the counters that must start at zero are cleared
// at the start of each call.
#include "snn_b200.h"
#include "b200_kernels.h"

#include <cuda_runtime.h>

#include <mutex>

namespace {

constexpr uint64_t kMaxNeurons = SNN_B200_NOALLOC_MAX_NEURONS;
constexpr uint64_t kCounterBytes = 256;
constexpr uint64_t kBitmapBytes = (kMaxNeurons / 32) * 4;
constexpr uint64_t kListBytes = kMaxNeurons * 4;
constexpr uint64_t kScratchBytes = kCounterBytes + kBitmapBytes + kListBytes;

// Fixed scratch: [counters 256 B | bitmap kMaxNeurons/32 words | spike list u32].
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

// In host code g_noalloc_scratch names a host-side stand-in, not device
// memory: its device address is looked up once per device (with that device
// current) and cached here, for the lifetime of the device's primary context
// (a caller that resets the device must not call this entry point again).
constexpr int kMaxDevices = 64;
std::mutex g_mu;
void *g_scratch_addr[kMaxDevices] = {};

bool aligned(const void *p, uintptr_t a) { return ((uintptr_t)p % a) == 0; }

}  // namespace

extern "C" snn_status_t snn_b200_step_noalloc(int device, void *stream, snn_size_t neuron_count,
                                              const snn_lif_params_t *lif, float decay, float *voltage,
                                              float *current, const float *external, uint32_t *refractory,
                                              uint8_t *spikes, const snn_size_t *row_ptr, const uint32_t *col_idx,
                                              const float *weights, float *next_current) {
    if (lif == nullptr || voltage == nullptr || current == nullptr || refractory == nullptr ||
        spikes == nullptr || row_ptr == nullptr || col_idx == nullptr || weights == nullptr ||
        next_current == nullptr || device < 0 || device >= kMaxDevices)
        return SNN_ERR_INVALID_ARGUMENT;
    if (neuron_count == 0 || neuron_count > kMaxNeurons)
        return SNN_ERR_INVALID_ARGUMENT;  // beyond the fixed scratch: use a context instead
    // 16-byte vector loads/stores on the neuron arrays and the edge arrays.
    if (!aligned(voltage, 16) || !aligned(current, 16) || !aligned(refractory, 16) || !aligned(spikes, 4) ||
        (external && !aligned(external, 16)) || !aligned(col_idx, 16) || !aligned(weights, 16) ||
        !aligned(row_ptr, 8))
        return SNN_ERR_INVALID_ARGUMENT;

    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess) return SNN_ERR_CUDA;
    if (prev != device && cudaSetDevice(device) != cudaSuccess) return SNN_ERR_CUDA;
    void *scratch = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        if (g_scratch_addr[device] == nullptr) {
            // First call on this device: resolve the array's device address
            // with this device current, and check the result.
            void *p = nullptr;
            if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) {
                if (prev != device) cudaSetDevice(prev);
                return SNN_ERR_CUDA;
            }
            g_scratch_addr[device] = p;
        }
        scratch = g_scratch_addr[device];
    }
    cudaStream_t s = (cudaStream_t)stream;
    auto *ctr = (b200::DevCounters *)scratch;
    auto *bitmap = (uint32_t *)((char *)scratch + kCounterBytes);
    auto *list = (uint32_t *)((char *)scratch + kCounterBytes + kBitmapBytes);
    const b200::LifArgs args{decay, lif->v_rest, lif->v_reset, lif->v_threshold, lif->input_scale,
                             lif->refractory_steps};
    snn_status_t st = SNN_OK;
    // The list counters must start at zero; the bitmap words of all n neurons
    // are rewritten by the LIF kernel, so they need no clearing.
    if (cudaMemsetAsync(ctr, 0, sizeof(b200::DevCounters), s) != cudaSuccess) st = SNN_ERR_CUDA;
    if (st == SNN_OK) {
        b200::launch_lif(s, device, neuron_count, args, voltage, current, external, refractory, spikes, bitmap, list,
                         32, 0, ctr, 0);
        if (cudaGetLastError() != cudaSuccess) st = SNN_ERR_CUDA;
    }
    if (st == SNN_OK) {
        b200::launch_propagate_push(s, device, list, 32, row_ptr, col_idx, 32, weights, next_current, ctr, 0, 1);
        if (cudaGetLastError() != cudaSuccess) st = SNN_ERR_CUDA;
    }
    if (prev != device) cudaSetDevice(prev);
    return st;
}
