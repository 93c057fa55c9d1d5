// Standalone gated RMSNorm (the reference's gated_rmsnorm plugin kernel):
//   y = round( w * round(o * rsqrt(mean(o^2) + eps)) * silu(z) )
// over rows of dv, fp32 math, fp16 or bf16 I/O. One warp per row; the row is
// held in registers between the reduction and the output pass.
// Semantics: gatedRmsNormKernel.cu:21-54 (fp16 only there); the prefill kernel
// fuses the same math as its epilogue, this entry serves unfused callers.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "gdn_prefill.h"

namespace gdn {

template <typename T>
__device__ __forceinline__ float to_f(T x);
template <>
__device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <typename T>
__device__ __forceinline__ T from_f(float x);
template <>
__device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

constexpr int RMS_THREADS = 256;
constexpr int RMS_MAXPER = 16;  // register-resident elements per lane (dv <= 512)

template <typename T>
__global__ void __launch_bounds__(RMS_THREADS) gated_rmsnorm_kernel(const T* __restrict__ o,
                                                                    const T* __restrict__ z,
                                                                    const T* __restrict__ w,
                                                                    T* __restrict__ y, int64_t rows,
                                                                    int dv, float eps) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * (RMS_THREADS / 32) + warp;
    if (row >= rows) return;
    const T* orow = o + row * dv;
    const T* zrow = z + row * dv;
    T* yrow = y + row * dv;
    float ov[RMS_MAXPER];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < RMS_MAXPER; ++i) {
        const int j = lane + 32 * i;
        ov[i] = (j < dv) ? to_f(orow[j]) : 0.f;
        ss = fmaf(ov[i], ov[i], ss);
    }
    for (int j = lane + 32 * RMS_MAXPER; j < dv; j += 32) {  // rows wider than the register tile
        const float x = to_f(orow[j]);
        ss = fmaf(x, x, ss);
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float rstd = rsqrtf(ss / (float)dv + eps);
#pragma unroll
    for (int i = 0; i < RMS_MAXPER; ++i) {
        const int j = lane + 32 * i;
        if (j < dv) {
            const float nb = to_f(from_f<T>(ov[i] * rstd));
            const float zf = to_f(zrow[j]);
            const float sg = zf * (1.f / (1.f + expf(-zf)));
            yrow[j] = from_f<T>((to_f(w[j]) * nb) * sg);
        }
    }
    for (int j = lane + 32 * RMS_MAXPER; j < dv; j += 32) {
        const float nb = to_f(from_f<T>(to_f(orow[j]) * rstd));
        const float zf = to_f(zrow[j]);
        const float sg = zf * (1.f / (1.f + expf(-zf)));
        yrow[j] = from_f<T>((to_f(w[j]) * nb) * sg);
    }
}

}  // namespace gdn

extern "C" cudaError_t gated_rmsnorm_forward(const void* o, const void* z, const void* w, void* y,
                                             int64_t rows, int dv, float eps, int dtype,
                                             cudaStream_t stream) {
    if (rows < 0 || dv <= 0 || (dtype != 0 && dtype != 1)) return cudaErrorInvalidValue;
    if (rows == 0) return cudaSuccess;
    if (!o || !z || !w || !y) return cudaErrorInvalidValue;
    const int64_t per_block = gdn::RMS_THREADS / 32;
    const int64_t blocks = (rows + per_block - 1) / per_block;
    if (blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
    if (dtype == 0)
        gdn::gated_rmsnorm_kernel<__half><<<(unsigned)blocks, gdn::RMS_THREADS, 0, stream>>>(
            (const __half*)o, (const __half*)z, (const __half*)w, (__half*)y, rows, dv, eps);
    else
        gdn::gated_rmsnorm_kernel<__nv_bfloat16><<<(unsigned)blocks, gdn::RMS_THREADS, 0, stream>>>(
            (const __nv_bfloat16*)o, (const __nv_bfloat16*)z, (const __nv_bfloat16*)w, (__nv_bfloat16*)y,
            rows, dv, eps);
    return cudaGetLastError();
}
