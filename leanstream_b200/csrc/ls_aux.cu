// Auxiliary sm_100a kernels of the backend:
//   * the tensor-parallel layer epilogue: after the fp32 partial outputs of
//     all ranks are summed (NCCL allreduce), round once to fp16 and add the
//     residual, as backends/triton/reduction.py:14-20 does on one GPU;
//   * a bounded device-side delay used to queue timed launches back to back.
#include <cuda_fp16.h>
#include <cerrno>
#include <stdint.h>
#include "ls_internal.h"

namespace lsb {
namespace {

__global__ void tp_epilogue_kernel(const float* __restrict__ y32, const __half* __restrict__ residual,
                                   __half* __restrict__ y, __half* __restrict__ hidden, uint32_t H) {
    for (uint32_t c = blockIdx.x * blockDim.x + threadIdx.x; c < H; c += gridDim.x * blockDim.x) {
        const __half y16 = __float2half_rn(y32[c]);
        if (y) y[c] = y16;
        if (hidden) hidden[c] = __float2half_rn(__half2float(residual[c]) + __half2float(y16));
    }
}

__global__ void spin_kernel(uint64_t ns) {
    uint64_t start, now;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(start));
    do {
        __nanosleep(1000);
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
    } while (now - start < ns);
}

}  // namespace
}  // namespace lsb

extern "C" {

int ls_b200_tp_epilogue(const float* y32, const void* residual, void* output, void* hidden_out, uint32_t hidden,
                        void* stream) {
    if (!y32 || !hidden || (hidden_out && !residual) || (!output && !hidden_out)) return EINVAL;
    const int threads = 256;
    int blocks = int((hidden + threads - 1) / threads);
    if (blocks > 64) blocks = 64;
    lsb::tp_epilogue_kernel<<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(
        y32, static_cast<const __half*>(residual), static_cast<__half*>(output), static_cast<__half*>(hidden_out),
        hidden);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : int(e);
}

int ls_b200_spin(uint64_t nanoseconds, void* stream) {
    if (nanoseconds > 100000000ull) return EINVAL;  // at most 100 ms
    lsb::spin_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(nanoseconds);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : int(e);
}

}  // extern "C"
