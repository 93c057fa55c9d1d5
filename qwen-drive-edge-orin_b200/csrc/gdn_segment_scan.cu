// Entry states of the segments of long sequences (deltanet_chunk_prefill_segmented).
//
// A run of chunks maps its entry state affinely: S_end = Phi S_start + A, where A is the
// run's final state from a zero entry state and Phi (d x d, acting on the key dimension) its
// final state from the identity with v = 0 (the chunk update S <- (e^{cL} I - K^T diag(e^{cL-c})
// W) S + K^T diag(e^{cL-c}) U is affine in S, and U vanishes with v). With a sequence cut into
// segments j = 0 .. n-1, the entry states follow by the scan S_0 = s0, S_{j+1} = Phi_j S_j + A_j.
//
// Columns of the state are independent under S <- Phi S + A, so each block owns a block of 8
// columns of one (sequence, v-head) and walks the segments in order: thread i computes row i of
// the new columns from row i of Phi (read from global memory, L1-cached) and the current
// columns (in shared memory, read as broadcasts). fp32 with two interleaved partial sums per
// output; the rounding of the scan stays below that of the kernels that produced A and Phi.
#include <cuda_runtime.h>
#include <stdint.h>

namespace gdn {

namespace {
constexpr int D = 128;  // head dim (state is D x D)
constexpr int CB = 8;   // state columns per block

// stt:   [B * nseg][2 HV][D][D]: A_j of head h at index h, Phi_j at index HV + h
// s0:    [B][HV][D][D] or null (zero entry state)
// entry: [B * nseg][HV][D][D] out: S_j, the entry state of segment j
__global__ void __launch_bounds__(D) segment_scan_kernel(const float* __restrict__ stt, const float* __restrict__ s0,
                                                         float* __restrict__ entry, int HV, int nseg) {
    __shared__ __align__(16) float cur[D][CB];
    const int i = threadIdx.x, c0 = blockIdx.x * CB, h = blockIdx.y, b = blockIdx.z;
    const size_t DD = (size_t)D * D;
    float s[CB];
#pragma unroll
    for (int c = 0; c < CB; ++c) s[c] = s0 ? s0[((size_t)b * HV + h) * DD + (size_t)i * D + c0 + c] : 0.f;
    for (int j = 0;; ++j) {
        float* out = entry + ((size_t)(b * nseg + j) * HV + h) * DD + (size_t)i * D + c0;
        *reinterpret_cast<float4*>(out) = make_float4(s[0], s[1], s[2], s[3]);
        *reinterpret_cast<float4*>(out + 4) = make_float4(s[4], s[5], s[6], s[7]);
        if (j + 1 >= nseg) break;
        __syncthreads();  // every thread is done reading the previous columns
#pragma unroll
        for (int c = 0; c < CB; ++c) cur[i][c] = s[c];
        __syncthreads();
        const size_t base = (size_t)(b * nseg + j) * 2 * HV;
        const float* A = stt + (base + h) * DD + (size_t)i * D + c0;
        const float* Phi = stt + (base + HV + h) * DD + (size_t)i * D;
        float a0[CB], a1[CB];
#pragma unroll
        for (int c = 0; c < CB; ++c) {
            a0[c] = A[c];
            a1[c] = 0.f;
        }
#pragma unroll 4
        for (int k = 0; k < D; k += 4) {
            const float4 ph = *reinterpret_cast<const float4*>(Phi + k);
            const float4 r0a = *reinterpret_cast<const float4*>(&cur[k][0]), r0b = *reinterpret_cast<const float4*>(&cur[k][4]);
            const float4 r1a = *reinterpret_cast<const float4*>(&cur[k + 1][0]), r1b = *reinterpret_cast<const float4*>(&cur[k + 1][4]);
            const float4 r2a = *reinterpret_cast<const float4*>(&cur[k + 2][0]), r2b = *reinterpret_cast<const float4*>(&cur[k + 2][4]);
            const float4 r3a = *reinterpret_cast<const float4*>(&cur[k + 3][0]), r3b = *reinterpret_cast<const float4*>(&cur[k + 3][4]);
            const float r0[CB] = {r0a.x, r0a.y, r0a.z, r0a.w, r0b.x, r0b.y, r0b.z, r0b.w};
            const float r1[CB] = {r1a.x, r1a.y, r1a.z, r1a.w, r1b.x, r1b.y, r1b.z, r1b.w};
            const float r2[CB] = {r2a.x, r2a.y, r2a.z, r2a.w, r2b.x, r2b.y, r2b.z, r2b.w};
            const float r3[CB] = {r3a.x, r3a.y, r3a.z, r3a.w, r3b.x, r3b.y, r3b.z, r3b.w};
#pragma unroll
            for (int c = 0; c < CB; ++c) {
                a0[c] = fmaf(ph.x, r0[c], a0[c]);
                a1[c] = fmaf(ph.y, r1[c], a1[c]);
                a0[c] = fmaf(ph.z, r2[c], a0[c]);
                a1[c] = fmaf(ph.w, r3[c], a1[c]);
            }
        }
#pragma unroll
        for (int c = 0; c < CB; ++c) s[c] = a0[c] + a1[c];
    }
}
}  // namespace

// Grid (D / CB column blocks, HV, B), D threads per block. stt, s0 and entry must be 16-byte aligned.
cudaError_t launch_segment_scan(const float* stt, const float* s0, float* entry, int B, int HV, int nseg,
                                cudaStream_t stream) {
    if (B <= 0 || HV <= 0 || nseg <= 0 || B > 65535 || HV > 65535) return cudaErrorInvalidValue;
    segment_scan_kernel<<<dim3(D / CB, HV, B), D, 0, stream>>>(stt, s0, entry, HV, nseg);
    return cudaGetLastError();
}

}  // namespace gdn
