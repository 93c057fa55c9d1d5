// Recurrent (decode) form of the gated delta rule: T tokens processed one
// after another against a state kept in registers, with the optional fused
// gated RMSNorm. The per-token update follows transformers
// torch_recurrent_gated_delta_rule (the decode path the reference leaves to
// stock Edge-LLM, export/patches/orin_text_engine/README.md:15):
//   S <- S e^{g_t};  kv = S^T k_t;  delta = (v_t - kv) beta_t;  S <- S + k_t delta^T;
//   o_t = S^T (q_t / sqrt(DK)).
// The step is memory-bound (the 64 KB state of each head is read and written
// once per call), so it runs on CUDA cores: one CTA per (sequence, v-head),
// thread (dv, part) holds S[dk][dv] for its 64 dk rows in registers; the dk
// reductions meet in shared memory.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "gdn_prefill.h"

namespace gdn {
namespace decode {

constexpr int HD = 128;
constexpr int NT = 256;

__global__ void __launch_bounds__(NT) gdn_decode_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
    const __nv_bfloat16* __restrict__ v, const float* __restrict__ g, const float* __restrict__ beta,
    const __nv_bfloat16* __restrict__ z, const __nv_bfloat16* __restrict__ w, float eps,
    __nv_bfloat16* __restrict__ out, float* state, int T, int HV, int HQK, float scale) {
    __shared__ float qs[HD], ks[HD], red[2][HD], nrm[8];
    const int tid = threadIdx.x, dv = tid & (HD - 1), part = tid >> 7;
    const int h = blockIdx.x, b = blockIdx.y;
    const int hq = h / (HV / HQK);
    float* S = state + ((size_t)b * HV + h) * HD * HD;
    float s[64];
#pragma unroll
    for (int j = 0; j < 64; ++j) s[j] = S[(size_t)(64 * part + j) * HD + dv];
    const bool gated = (z != nullptr);
    const float wv = gated ? __bfloat162float(w[dv]) : 0.f;

    for (int t = 0; t < T; ++t) {
        const size_t tok = (size_t)b * T + t;
        if (tid < HD) {
            qs[tid] = __bfloat162float(q[(tok * HQK + hq) * HD + tid]) * scale;
        } else {
            ks[tid - HD] = __bfloat162float(k[(tok * HQK + hq) * HD + (tid - HD)]);
        }
        const float decay = expf(g[tok * HV + h]);
        const float bt = beta[tok * HV + h];
        const float vt = __bfloat162float(v[(tok * HV + h) * HD + dv]);
        __syncthreads();
        float kv = 0.f;
#pragma unroll
        for (int j = 0; j < 64; ++j) {
            s[j] *= decay;
            kv = fmaf(s[j], ks[64 * part + j], kv);
        }
        red[part][dv] = kv;
        __syncthreads();
        const float delta = (vt - (red[0][dv] + red[1][dv])) * bt;
        float o = 0.f;
#pragma unroll
        for (int j = 0; j < 64; ++j) {
            s[j] = fmaf(ks[64 * part + j], delta, s[j]);
            o = fmaf(s[j], qs[64 * part + j], o);
        }
        __syncthreads();  // red[] reads done
        red[part][dv] = o;
        __syncthreads();
        __nv_bfloat16* dst = out + (tok * HV + h) * HD + dv;
        if (!gated) {
            if (part == 0) *dst = __float2bfloat16_rn(red[0][dv] + red[1][dv]);
        } else {
            // y = bf16( w * bf16(o * rsqrt(mean(o^2) + eps)) * silu(z) ), o rounded to bf16 first
            const float ob = __bfloat162float(__float2bfloat16_rn(red[0][dv] + red[1][dv]));
            float sq = (part == 0) ? ob * ob : 0.f;
#pragma unroll
            for (int off = 16; off; off >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, off);
            if ((tid & 31) == 0) nrm[tid >> 5] = sq;
            __syncthreads();
            const float ss = nrm[0] + nrm[1] + nrm[2] + nrm[3];
            const float rstd = rsqrtf(ss / (float)HD + eps);
            if (part == 0) {
                const float nb = __bfloat162float(__float2bfloat16_rn(ob * rstd));
                const float zf = __bfloat162float(z[(tok * HV + h) * HD + dv]);
                *dst = __float2bfloat16_rn((wv * nb) * (zf / (1.f + expf(-zf))));
            }
        }
        __syncthreads();  // qs/ks/red/nrm reused by the next token
    }
#pragma unroll
    for (int j = 0; j < 64; ++j) S[(size_t)(64 * part + j) * HD + dv] = s[j];
}

}  // namespace decode
}  // namespace gdn

extern "C" cudaError_t deltanet_recurrent_decode(const void* q, const void* k, const void* v, const float* g,
                                                 const float* beta, const void* z, const void* norm_w, float eps,
                                                 void* out, float* state, int B, int T, int HV, int HQK, int DK,
                                                 int DV, cudaStream_t stream) {
    if (DK != gdn::decode::HD || DV != gdn::decode::HD) return cudaErrorInvalidValue;
    if (HQK <= 0 || HV <= 0 || HV % HQK != 0 || B < 0 || T < 0 || HV > 65535 || B > 65535) return cudaErrorInvalidValue;
    if ((z == nullptr) != (norm_w == nullptr)) return cudaErrorInvalidValue;
    if (B == 0 || T == 0) return cudaSuccess;
    if (!q || !k || !v || !g || !beta || !out || !state) return cudaErrorInvalidValue;
    gdn::decode::gdn_decode_kernel<<<dim3(HV, B), gdn::decode::NT, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
        static_cast<const __nv_bfloat16*>(v), g, beta, static_cast<const __nv_bfloat16*>(z),
        static_cast<const __nv_bfloat16*>(norm_w), eps, static_cast<__nv_bfloat16*>(out), state, T, HV, HQK,
        1.0f / sqrtf((float)DK));
    return cudaGetLastError();
}
