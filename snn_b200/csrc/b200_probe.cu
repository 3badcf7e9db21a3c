// Diagnostic: the L2 reduction ceiling the push propagation runs against.
//
// The push kernel issues one red.global.add.f32 per synaptic event into the
// L2-resident target currents; its throughput is bounded by how many such
// reductions to scattered addresses the L2 serves per second, not by HBM
// bytes. This probe measures that ceiling on the current device with the
// push kernel's access pattern: `events` reductions of 1.0f into uniformly
// random slots of a `targets`-float array (the targets drawn with splitmix64,
// read with 16-byte loads, four reductions per load), timed with CUDA events.
#include "snn_b200.h"
#include "b200_kernels.h"

#include <cuda_runtime.h>

namespace {

__global__ void probe_fill_targets(uint32_t *idx, uint64_t events, uint64_t targets, uint64_t seed) {
    const uint64_t stride = (uint64_t)blockDim.x * gridDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < events; i += stride) {
        uint64_t z = seed + (i + 1) * 0x9e3779b97f4a7c15ull;
        z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
        z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
        idx[i] = (uint32_t)((z ^ (z >> 31)) % targets);
    }
}

__global__ void __launch_bounds__(256) probe_red_kernel(const uint4 *__restrict__ idx, uint64_t vecs,
                                                        float *__restrict__ dst) {
    const uint64_t stride = (uint64_t)blockDim.x * gridDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < vecs; i += stride) {
        const uint4 v = __ldcs(idx + i);
        atomicAdd(dst + v.x, 1.0f);
        atomicAdd(dst + v.y, 1.0f);
        atomicAdd(dst + v.z, 1.0f);
        atomicAdd(dst + v.w, 1.0f);
    }
}

}  // namespace

extern "C" snn_status_t snn_b200_probe_red_rate(int device, uint64_t targets, uint64_t events, uint32_t repeats,
                                                double *out_reds_per_s) {
    if (out_reds_per_s == nullptr || targets == 0 || targets > 0xffffffffull || events < 4 || repeats == 0)
        return SNN_ERR_INVALID_ARGUMENT;
    *out_reds_per_s = 0.0;
    if (cudaSetDevice(device) != cudaSuccess) return SNN_ERR_CUDA;
    const uint64_t vecs = events / 4;
    float *dst = nullptr;
    uint32_t *idx = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    snn_status_t st = SNN_OK;
    if (cudaMalloc(&dst, targets * 4) != cudaSuccess || cudaMalloc(&idx, vecs * 16) != cudaSuccess ||
        cudaEventCreate(&e0) != cudaSuccess || cudaEventCreate(&e1) != cudaSuccess)
        st = SNN_ERR_OUT_OF_MEMORY;
    if (st == SNN_OK) {
        const int grid = b200::sm_count(device) * 8;
        cudaMemset(dst, 0, targets * 4);
        probe_fill_targets<<<grid, 256>>>(idx, vecs * 4, targets, 12345);
        probe_red_kernel<<<grid, 256>>>((const uint4 *)idx, vecs, dst);  // warm-up
        cudaEventRecord(e0);
        for (uint32_t r = 0; r < repeats; ++r) probe_red_kernel<<<grid, 256>>>((const uint4 *)idx, vecs, dst);
        cudaEventRecord(e1);
        float ms = 0.0f;
        if (cudaEventSynchronize(e1) != cudaSuccess || cudaEventElapsedTime(&ms, e0, e1) != cudaSuccess || ms <= 0)
            st = SNN_ERR_CUDA;
        else
            *out_reds_per_s = (double)vecs * 4.0 * repeats / (ms * 1e-3);
    }
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    if (idx) cudaFree(idx);
    if (dst) cudaFree(dst);
    cudaGetLastError();
    return st;
}
