// Entry states of the segments of long sequences (deltanet_chunk_prefill_segmented).
//
// A run of chunks maps its entry state affinely: S_end = Phi S_start + A, where A is the
// run's final state from a zero entry state and Phi (d x d, acting on the key dimension) its
// final state from the identity with v = 0 (the chunk update S <- (e^{cL} I - K^T diag(e^{cL-c})
// W) S + K^T diag(e^{cL-c}) U is affine in S, and U vanishes with v). With a sequence cut into
// segments j = 0 .. n-1, the entry states follow by the scan S_0 = s0, S_{j+1} = Phi_j S_j + A_j
// (the last segment's maps are not needed, and the state pass does not form them).
//
// Columns of the state are independent under S <- Phi S + A, so each block owns a block of 4
// columns of one (sequence, v-head) and walks the segments in order; thread i computes row i of
// the new columns. The state pass stores Phi transposed (PhiT[k][i] = Phi[i][k]), so that a step
// reads, for each k, one float of PhiT row k per thread (consecutive threads, consecutive banks)
// and the 4 current values of row k as a broadcast; loads of 16 values of k go ahead of their
// products. A step is bound by the shared-memory pipe (the broadcasts cost a full pass each), so
// the blocks are narrow: 32 per (sequence, head). The map and the block's columns of A of a step
// are copied into shared memory two steps ahead (16-byte cp.async copies, many in flight per
// thread; three buffers), so that the serial loop waits on no global load. fp32; the rounding of
// the scan stays below that of the kernels that produced A and Phi.
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

namespace gdn {

namespace {
constexpr int D = 128;        // head dim (state is D x D)
constexpr int CB = 4;         // state columns per block
constexpr int NT = D;         // threads: one per row
constexpr int KB = 16;        // values of k whose loads go ahead of their products
constexpr int NBUF = 3;       // map buffers (copies in flight: NBUF - 1 steps ahead of the step computing)
constexpr uint32_t MAP_BYTES = D * D * 4;
constexpr uint32_t SLICE_BYTES = D * CB * 4;  // a block's columns of A (or of the current state)
constexpr uint32_t SCAN_SMEM = NBUF * (MAP_BYTES + SLICE_BYTES) + SLICE_BYTES;
static_assert(SCAN_SMEM <= 232448, "exceeds the 227 KB per-block shared memory limit");

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(reinterpret_cast<uint64_t>(src))
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// wait until at most N of this thread's copy groups are pending (groups complete in order)
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// stt:   [B * nmap][2 HV][D][D], nmap = nseg - 1: A_j of head h at index h, PhiT_j at HV + h
// s0:    [B][HV][D][D] or null (zero entry state)
// entry: [B * nseg][HV][D][D] out: S_j, the entry state of segment j
__global__ void __launch_bounds__(NT) segment_scan_kernel(const float* __restrict__ stt, const float* __restrict__ s0,
                                                          float* __restrict__ entry, int HV, int nseg) {
    extern __shared__ __align__(16) uint8_t smem[];
    float* abuf = reinterpret_cast<float*>(smem + NBUF * MAP_BYTES);      // NBUF x [D][CB]
    float* cur = reinterpret_cast<float*>(smem + NBUF * (MAP_BYTES + SLICE_BYTES));  // [D][CB]
    const uint32_t sb = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    const int i = threadIdx.x, c0 = blockIdx.x * CB, h = blockIdx.y, b = blockIdx.z;
    const size_t DD = (size_t)D * D;
    const int nmap = nseg - 1;
    // the maps come from the previous launch (the state pass): nothing global is read before this
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // every thread copies 32 of the map's 4096 16-byte pieces and its row of A's columns, and
    // commits one group per step (an empty group past the last map, so that the wait below
    // counts the same every step)
    auto copy_step = [&](int j) {
        if (j < nmap) {
            const float* base = stt + (size_t)(b * nmap + j) * 2 * HV * DD;
            const float* src = base + (size_t)(HV + h) * DD;
            const uint32_t dst = sb + (uint32_t)(j % NBUF) * MAP_BYTES;
#pragma unroll
            for (int u = 0; u < (int)(MAP_BYTES / 16) / NT; ++u) {
                const int piece = u * NT + i;
                cp_async16(dst + 16u * (uint32_t)piece, src + 4 * piece);
            }
            cp_async16(sb + NBUF * MAP_BYTES + (uint32_t)(j % NBUF) * SLICE_BYTES + 16u * (uint32_t)i,
                       base + (size_t)h * DD + (size_t)i * D + c0);
        }
        cp_async_commit();
    };
    for (int j = 0; j < NBUF - 1; ++j) copy_step(j);
    float4 s = s0 ? *reinterpret_cast<const float4*>(s0 + ((size_t)b * HV + h) * DD + (size_t)i * D + c0)
                  : make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0;; ++j) {
        *reinterpret_cast<float4*>(entry + ((size_t)(b * nseg + j) * HV + h) * DD + (size_t)i * D + c0) = s;
        if (j >= nmap) break;
        copy_step(j + NBUF - 1);  // into the buffers that step j - 1 read (every thread passed the barrier below)
        *reinterpret_cast<float4*>(cur + i * CB) = s;
        cp_async_wait<NBUF - 1>();  // this thread's pieces of step j have landed
        __syncthreads();            // everyone's pieces, and the current columns, are visible
        const float* phiT = reinterpret_cast<const float*>(smem + (size_t)(j % NBUF) * MAP_BYTES);
        const float4 a = *reinterpret_cast<const float4*>(abuf + (j % NBUF) * D * CB + i * CB);
        float a0[CB] = {a.x, a.y, a.z, a.w}, a1[CB] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
        for (int k0 = 0; k0 < D; k0 += KB) {
            float p[KB];
            float4 r[KB];
#pragma unroll
            for (int u = 0; u < KB; ++u) p[u] = phiT[(k0 + u) * D + i];
#pragma unroll
            for (int u = 0; u < KB; ++u) r[u] = *reinterpret_cast<const float4*>(cur + (k0 + u) * CB);
#pragma unroll
            for (int u = 0; u < KB; u += 2) {
                a0[0] = fmaf(p[u], r[u].x, a0[0]);
                a0[1] = fmaf(p[u], r[u].y, a0[1]);
                a0[2] = fmaf(p[u], r[u].z, a0[2]);
                a0[3] = fmaf(p[u], r[u].w, a0[3]);
                a1[0] = fmaf(p[u + 1], r[u + 1].x, a1[0]);
                a1[1] = fmaf(p[u + 1], r[u + 1].y, a1[1]);
                a1[2] = fmaf(p[u + 1], r[u + 1].z, a1[2]);
                a1[3] = fmaf(p[u + 1], r[u + 1].w, a1[3]);
            }
        }
        s = make_float4(a0[0] + a1[0], a0[1] + a1[1], a0[2] + a1[2], a0[3] + a1[3]);
        __syncthreads();  // every thread is done with this step's buffers and the current columns
    }
    cp_async_wait<0>();  // (only empty groups can be pending here)
}
}  // namespace

// Grid (D / CB column blocks, HV, B), D threads per block, launched as a programmatic dependent
// of the state pass. stt, s0 and entry must be 16-byte aligned.
cudaError_t launch_segment_scan(const float* stt, const float* s0, float* entry, int B, int HV, int nseg,
                                cudaStream_t stream) {
    if (B <= 0 || HV <= 0 || nseg <= 0 || B > 65535 || HV > 65535) return cudaErrorInvalidValue;
    static std::atomic<bool> attr_set[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev].load(std::memory_order_acquire)) {  // idempotent: threads that race here set the same value
        e = cudaFuncSetAttribute(segment_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SCAN_SMEM);
        if (e != cudaSuccess) return e;
        attr_set[dev].store(true, std::memory_order_release);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(D / CB, HV, B);
    cfg.blockDim = dim3(NT, 1, 1);
    cfg.dynamicSmemBytes = SCAN_SMEM;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, segment_scan_kernel, stt, s0, entry, HV, nseg);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

}  // namespace gdn
