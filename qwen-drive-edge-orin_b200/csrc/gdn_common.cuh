// Device helpers shared by the prefill kernels: launch parameters, 128-byte
// swizzle addressing of bf16 tiles, bf16 hi/lo splitting, fast exp2 /
// reciprocal, and the 64x64 unit-lower-triangular inverse.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "sm100_ptx.cuh"

namespace gdn {

constexpr int CS = 64;         // chunk length (tokens)
constexpr int HD = 128;        // head dim (DK = DV)
constexpr int LSTRIDE = 68;    // fp32 row stride of the L / T scratch (16-byte aligned rows)
// Poll limit of every mbarrier wait. A poll is a try_wait (which may suspend the thread for a
// hardware-chosen time) and, after the first 4096, a 64 ns sleep: measured on B200, 2^22 polls
// took 17 s, so 2^18 gives up after about one second.
constexpr uint32_t WAIT_ITERS = 1u << 18;

struct Params {
    CUtensorMap tm_q, tm_k, tm_v, tm_z;
    const float* g;
    const float* beta;
    const __nv_bfloat16* w;        // norm weight [128] (gated only)
    const float* s0;               // [NSEQ, HV, 128, 128] or null
    float* sf;                     // [NSEQ, HV, 128, 128]
    __nv_bfloat16* out;            // o or y, [B, T, HV, 128] / [1, T, HV, 128]
    const int* cu_seqlens;         // varlen offsets or null
    unsigned int* status;          // workspace status word
    float* dbg;                    // debug records or null
    int T;                         // tokens per batch row (fixed) / total tokens (varlen)
    int HV, HQK;
    int max_nc;                    // chunks of the longest sequence (debug indexing)
    float scale;                   // 1/sqrt(DK)
    float eps;
    int gated;
    // Pre-stage mode (the reference's TRT adapter inputs): q/k/v/z/w and the
    // output are fp16, q/k arrive un-normalised (L2-normalised here in fp32 and
    // rounded to bf16), v is rounded to bf16, and the gates are computed from
    // a, b (fp16 [.., HV]), A_log (fp32 [HV]) and dt_bias (fp16 [HV]).
    int prestage;
    const __half* ga;
    const __half* gb;
    const float* A_log;
    const __half* dt_bias;
    // Test hook: the v-tile load of this chunk is never issued (-1: every load is issued), so
    // that the bounded wait for it runs out and the abort path runs. Set only by
    // deltanet_test_withheld_load.
    int withhold_v_chunk;
    // Segments of long sequences (deltanet_chunk_prefill_segmented; the kernels' segmented instantiations).
    // seg_chunks > 0: block z indexes (sequence b, segment j) = (z / seg_per_seq, z % seg_per_seq)
    // and covers tokens [j * seg_chunks * 64, min((j + 1) * seg_chunks * 64, T)) of batch row b.
    int seg_chunks, seg_per_seq;
    // State pass of a segmented call (grid y = 2 HV): blocks with blockIdx.y >= HV run v-head
    // blockIdx.y - HV from the identity state with v = 0 (the cluster-split kernel reads it through
    // tm_v0, a map over a zero tile, every other box out of bounds, so every load is zero; the
    // one-CTA kernel loads no v); the others run from a zero state (s0 null). Each block writes its
    // final state at index (z, blockIdx.y) of sf, the identity runs' transposed (the scan's layout).
    CUtensorMap tm_v0;
    // Output pass of a segmented call: only the last segment of each sequence writes its final
    // state, at sf[b] (the other segments' final states are the next segments' entry states).
    int sf_last_only;
    // One-CTA kernel's segmented passes: a record of T' and W^T hi/lo tiles (48 KB, the
    // shared-memory tile layout) per chunk of every (sequence, segment, head), written by the
    // zero-state runs and read by the identity runs and the output pass (which then form no
    // triangular inverse of their own); seg_total = segments per sequence (record indexing).
    uint8_t* wbuf;
    int seg_total;
};

// Byte offset of bf16 element (row, col) in a 128B-swizzled tile whose panels
// hold `rows` rows each.
__device__ __forceinline__ uint32_t sw_off(int row, int col, int rows) {
    return (uint32_t)((col >> 6) * rows * 128 + row * 128 + ((((col & 63) >> 3) ^ (row & 7)) << 4) +
                      ((col & 7) << 1));
}
// Byte offset of fp32 element group [4j, 4j+4) of row `row` in the [64][128] fp32 gate
// tile: the 16-byte chunk index is XOR-swizzled with the row inside each group of 8.
__device__ __forceinline__ uint32_t gate_chunk(int row, int j) {
    return (uint32_t)(row * 512 + (((j & ~7) | ((j ^ row) & 7)) << 4));
}
// Byte offset of the 16-byte chunk holding cols [8*ch, 8*ch+8) of `row`.
__device__ __forceinline__ uint32_t sw_chunk(int row, int ch, int rows) {
    return (uint32_t)((ch >> 3) * rows * 128 + row * 128 + (((ch & 7) ^ (row & 7)) << 4));
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ float bf16r(float x) {
    return __bfloat162float(__float2bfloat16_rn(x));
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
                 "r"(d)
                 : "memory");
}
__device__ __forceinline__ void ld_shared_v4(uint32_t addr, uint32_t& a, uint32_t& b, uint32_t& c,
                                             uint32_t& d) {
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(a), "=r"(b), "=r"(c), "=r"(d)
                 : "r"(addr)
                 : "memory");
}
__device__ __forceinline__ float ex2f(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float rcpf(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
// Read-only global loads issued where they are written: a prefetch for a later chunk must
// not be moved by the compiler down to its first use, where its latency would be exposed.
__device__ __forceinline__ float ldg_early(const float* p) {
    float v;
    asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ __half ldg_early(const __half* p) {
    unsigned short v;
    asm volatile("ld.global.nc.b16 %0, [%1];" : "=h"(v) : "l"(p));
    return __ushort_as_half(v);
}
constexpr float LOG2E = 1.4426950408889634f;

// Split two fp32 values into packed bf16 hi parts and packed bf16 lo parts
// (x = hi + lo to ~16 mantissa bits).
// ---------------------------------------------------------------------------
// Packed fp32 pairs: sm_100 runs add / mul / fma on the two fp32 halves of a 64-bit
// register pair in one instruction (PTX .f32x2, round-to-nearest like the scalar forms),
// which halves the instruction count of the element-wise steps.
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t r, float& a, float& b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

// bf16 hi/lo split of two values: hi = bf16(x), lo = bf16(x - hi).
__device__ __forceinline__ void split2(float a, float b, uint32_t& hi, uint32_t& lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = pack_bf16(a - __low2float(h), b - __high2float(h));
}
// The same split with the two residuals in one packed subtraction (fewer instructions,
// but the packed operands want register pairs: for code with registers to spare).
__device__ __forceinline__ void split2x(float a, float b, uint32_t& hi, uint32_t& lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    float ra, rb;
    f2_unpack(f2_sub(f2_pack(a, b), f2_pack(__uint_as_float(hi << 16), __uint_as_float(hi & 0xFFFF0000u))), ra, rb);
    lo = pack_bf16(ra, rb);
}

// Write 8 consecutive fp32 values as bf16 hi (and optionally lo) parts into a
// 16-byte chunk of two tiles.
__device__ __forceinline__ void put8_split(uint32_t hi_addr, uint32_t lo_addr, const float* x,
                                           bool want_lo) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) split2x(x[2 * i], x[2 * i + 1], h[i], l[i]);
    st_shared_v4(hi_addr, h[0], h[1], h[2], h[3]);
    if (want_lo) st_shared_v4(lo_addr, l[0], l[1], l[2], l[3]);
}

// ---------------------------------------------------------------------------
// T = (I + L)^-1 for a 64x64 strictly-lower L held in Ls (stride 68), in place.
//   A: the four 16x16 diagonal blocks by forward substitution (one warp each,
//      lane = column, column in registers);
//   B/C: 32x32 halves: T_10 = -(T_11 L_10) T_00 and T_32 = -(T_33 L_32) T_22;
//   D/E: T_[32:,:32] = -(T_[32:,32:] L_[32:,:32]) T_[:32,:32].
// The block products B-E are small (16x16x16 and 32x32x32) and sit on a chain of
// dependent steps. Two implementations, chosen by the template flag:
//   kTensorProducts = true: warp-level m16n8k8 tf32 tensor-core products with fp32
//     operands split in two tf32 terms (a = a_hi + a_lo; a b ~ a_hi b_hi + a_hi b_lo +
//     a_lo b_hi, the "3xTF32" scheme, about fp32 accuracy), one 16x8 output tile per
//     warp; X holds 1152 floats (rows of 36, conflict-free fragment loads).
//   kTensorProducts = false: CUDA-core products with 16-byte loads, register-blocked 1x4
//     (B, C) and 2x4 over split halves of the m range (D, E); X holds 2624 floats.
// Both skip the tiles or terms that the triangular factors make zero.
__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ void fma4(float4& acc, float a, const float4& b) {
    acc.x = fmaf(a, b.x, acc.x);
    acc.y = fmaf(a, b.y, acc.y);
    acc.z = fmaf(a, b.z, acc.z);
    acc.w = fmaf(a, b.w, acc.w);
}

namespace tf32x3 {
__device__ __forceinline__ uint32_t round_tf32(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return r;
}
__device__ __forceinline__ void split(float x, uint32_t& hi, uint32_t& lo) {
    hi = round_tf32(x);
    lo = round_tf32(x - __uint_as_float(hi));
}
// d += a b for one m16n8k8 tile (row-major A fragment, column-major B fragment)
__device__ __forceinline__ void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// Accumulators of one warp's 16x8 tile: main (hi*hi) and correction terms, two sets
// alternating by k-step so that consecutive products do not wait on each other.
struct Tile {
    float m[2][4], c[2][4];
    __device__ __forceinline__ Tile() {
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) m[i][j] = c[i][j] = 0.f;
    }
    // += A (16x8, element (r, k) at A[r * lda + k]) * B (8x8, element (k, n) at B[k * ldb + n])
    __device__ __forceinline__ void step(int par, const float* A, int lda, const float* B, int ldb, int lane) {
        const int g = lane >> 2, t = lane & 3;
        uint32_t ah[4], al[4], bh0, bl0, bh1, bl1;
        split(A[g * lda + t], ah[0], al[0]);
        split(A[(g + 8) * lda + t], ah[1], al[1]);
        split(A[g * lda + t + 4], ah[2], al[2]);
        split(A[(g + 8) * lda + t + 4], ah[3], al[3]);
        split(B[t * ldb + g], bh0, bl0);
        split(B[(t + 4) * ldb + g], bh1, bl1);
        mma(c[par], al, bh0, bh1);
        mma(m[par], ah, bh0, bh1);
        mma(c[par], ah, bl0, bl1);
    }
    // C (element (r, n) at C[r * ldc + n]) = s * tile
    __device__ __forceinline__ void store(float* C, int ldc, float s, int lane) const {
        const int g = lane >> 2, t = lane & 3;
        float d[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) d[j] = s * ((m[0][j] + m[1][j]) + (c[0][j] + c[1][j]));
        *reinterpret_cast<float2*>(C + g * ldc + 2 * t) = make_float2(d[0], d[1]);
        *reinterpret_cast<float2*>(C + (g + 8) * ldc + 2 * t) = make_float2(d[2], d[3]);
    }
};
}  // namespace tf32x3

// `idle(phase)` runs on threads 128-255 during phases A, B and C (phase = 0, 1, 2),
// which use only threads 0-127. `sync()` is the barrier over the 256 threads taking
// part (a block-wide __syncthreads, or a named barrier when other warps of the
// block do different work).
template <bool kTensorProducts, typename Idle, typename Sync>
__device__ __forceinline__ void invert_unit_lower(float* Ls, float* X, int tid, Idle&& idle, Sync&& sync) {
    constexpr int XS = 36;
    const int warp = tid >> 5, lane = tid & 31;
    if (tid >= 128) idle(0);
    // A: diagonal blocks
    if (warp < 4 && lane < 16) {
        const int b = warp, c = lane;
        const float* Lb = Ls + (16 * b) * LSTRIDE + 16 * b;
        float t[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            float a0 = (i == c) ? 1.f : 0.f, a1 = 0.f;
#pragma unroll
            for (int j = 0; j + 1 < i; j += 2) {
                a0 = fmaf(-Lb[i * LSTRIDE + j], t[j], a0);
                a1 = fmaf(-Lb[i * LSTRIDE + j + 1], t[j + 1], a1);
            }
            if (i & 1) a0 = fmaf(-Lb[i * LSTRIDE + i - 1], t[i - 1], a0);
            t[i] = a0 + a1;
        }
        __syncwarp(0x0000ffffu);
        float* Tb = Ls + (16 * b) * LSTRIDE + 16 * b;
#pragma unroll
        for (int i = 0; i < 16; ++i) Tb[i * LSTRIDE + c] = t[i];
    }
    sync();
    if constexpr (kTensorProducts) {
        // B: X_p = T_rr L_rc, 16x16 (p = 0: r = 16, c = 0; p = 1: r = 48, c = 32); warp = (p, n-tile)
        if (tid >= 128) idle(1);
        if (warp < 4) {
            const int pp = warp >> 1, nt = warp & 1, r0 = 16 + 32 * pp, c0 = 32 * pp;
            tf32x3::Tile acc;
    #pragma unroll
            for (int ks = 0; ks < 2; ++ks)
                acc.step(ks, Ls + r0 * LSTRIDE + r0 + 8 * ks, LSTRIDE, Ls + (r0 + 8 * ks) * LSTRIDE + c0 + 8 * nt, LSTRIDE,
                         lane);
            acc.store(X + pp * 16 * XS + 8 * nt, XS, 1.f, lane);
        }
        sync();
        // C: T_rc = -X_p T_cc (T_cc[k][n] = 0 for k < n: n-tile 1 skips k-step 0)
        if (tid >= 128) idle(2);
        if (warp < 4) {
            const int pp = warp >> 1, nt = warp & 1, r0 = 16 + 32 * pp, c0 = 32 * pp;
            tf32x3::Tile acc;
    #pragma unroll
            for (int ks = 0; ks < 2; ++ks)
                if (ks >= nt)
                    acc.step(ks, X + pp * 16 * XS + 8 * ks, XS, Ls + (c0 + 8 * ks) * LSTRIDE + c0 + 8 * nt, LSTRIDE, lane);
            acc.store(Ls + r0 * LSTRIDE + c0 + 8 * nt, LSTRIDE, -1.f, lane);
        }
        sync();
        // D: X2 = T_[32:,32:] L_[32:,:32] -> X (B's products are dead); rows 0-15 of T_[32:,32:]
        // are zero beyond column 15. warp = (m-tile, n-tile)
        {
            const int mt = warp >> 2, nt = warp & 3;
            tf32x3::Tile acc;
    #pragma unroll
            for (int ks = 0; ks < 4; ++ks)
                if (mt == 1 || ks < 2)
                    acc.step(ks & 1, Ls + (32 + 16 * mt) * LSTRIDE + 32 + 8 * ks, LSTRIDE,
                             Ls + (32 + 8 * ks) * LSTRIDE + 8 * nt, LSTRIDE, lane);
            acc.store(X + 16 * mt * XS + 8 * nt, XS, 1.f, lane);
        }
        sync();
        // E: T_[32:,:32] = -X2 T_[:32,:32] (T_[:32,:32][k][n] = 0 for k < n)
        {
            const int mt = warp >> 2, nt = warp & 3;
            tf32x3::Tile acc;
    #pragma unroll
            for (int ks = 0; ks < 4; ++ks)
                if (ks >= nt)
                    acc.step(ks & 1, X + 16 * mt * XS + 8 * ks, XS, Ls + (8 * ks) * LSTRIDE + 8 * nt, LSTRIDE, lane);
            acc.store(Ls + (32 + 16 * mt) * LSTRIDE + 8 * nt, LSTRIDE, -1.f, lane);
        }
        sync();
    } else {
        // B: X[0:256] = T_11 L_10, X[256:512] = T_33 L_32   (16x16 each, stride 16).
        // Terms above the diagonal of T_rr are stored zeros, so every unit runs the
        // full 16-term range in groups of four with its loads issued together.
        if (tid >= 128) idle(1);
        if (tid < 128) {
            const int blk = tid >> 6, i = (tid >> 2) & 15, j0 = (tid & 3) * 4;
            const int r0 = 16 + 32 * blk, c0 = 32 * blk;  // T_rr at (r0, r0), L block at (r0, c0)
            float4 acc0 = make_float4(0.f, 0.f, 0.f, 0.f), acc1 = acc0;
            const float* trow = Ls + (r0 + i) * LSTRIDE + r0;
    #pragma unroll
            for (int m0 = 0; m0 < 16; m0 += 4) {
                const float4 t4 = ld4(trow + m0);
                const float4 b0 = ld4(Ls + (r0 + m0) * LSTRIDE + c0 + j0), b1 = ld4(Ls + (r0 + m0 + 1) * LSTRIDE + c0 + j0);
                const float4 b2 = ld4(Ls + (r0 + m0 + 2) * LSTRIDE + c0 + j0), b3 = ld4(Ls + (r0 + m0 + 3) * LSTRIDE + c0 + j0);
                fma4(acc0, t4.x, b0); fma4(acc1, t4.y, b1); fma4(acc0, t4.z, b2); fma4(acc1, t4.w, b3);
            }
            *reinterpret_cast<float4*>(X + blk * 256 + i * 16 + j0) =
                make_float4(acc0.x + acc1.x, acc0.y + acc1.y, acc0.z + acc1.z, acc0.w + acc1.w);
        }
        sync();
        // C: T_10 = -X0 T_00 -> rows 16-31, cols 0-15; T_32 = -X1 T_22 -> rows 48-63, cols 32-47
        if (tid >= 128) idle(2);
        if (tid < 128) {
            const int blk = tid >> 6, i = (tid >> 2) & 15, j0 = (tid & 3) * 4;
            const int d0 = 32 * blk;  // T_ss at (d0, d0)
            float4 acc0 = make_float4(0.f, 0.f, 0.f, 0.f), acc1 = acc0;
            const float* xrow = X + blk * 256 + i * 16;
    #pragma unroll
            for (int m0 = 0; m0 < 16; m0 += 4) {
                const float4 x4 = ld4(xrow + m0);
                const float4 b0 = ld4(Ls + (d0 + m0) * LSTRIDE + d0 + j0), b1 = ld4(Ls + (d0 + m0 + 1) * LSTRIDE + d0 + j0);
                const float4 b2 = ld4(Ls + (d0 + m0 + 2) * LSTRIDE + d0 + j0), b3 = ld4(Ls + (d0 + m0 + 3) * LSTRIDE + d0 + j0);
                fma4(acc0, x4.x, b0); fma4(acc1, x4.y, b1); fma4(acc0, x4.z, b2); fma4(acc1, x4.w, b3);
            }
            *reinterpret_cast<float4*>(Ls + (d0 + 16 + i) * LSTRIDE + d0 + j0) =
                make_float4(-(acc0.x + acc1.x), -(acc0.y + acc1.y), -(acc0.z + acc1.z), -(acc0.w + acc1.w));
        }
        sync();
        // D: X2 = T_[32:,32:] L_[32:,:32], stored transposed: X2T[j][i] at X[512 + 34 j + i]. A thread
        // takes a 2x4 tile (rows 2rp, 2rp+1 of T_[32:,32:], columns 4cg..4cg+3) over half of the m
        // range (threads 128-255 the upper half, partial sums handed over in X[1600 + 8t]); warp w of
        // a half holds rows 8w..8w+7 and stops where T_[32:,32:] is zero (m > row), warp-uniformly.
        {
            const int kh = tid >> 7, t = tid & 127, rp = t >> 3, cg = t & 7, i0 = 2 * rp, j0 = 4 * cg;
            const int w8 = (t >> 5) * 8;
            const int mlo = kh ? 16 : 0, mhi = kh ? w8 + 8 : (w8 + 8 < 16 ? w8 + 8 : 16);
            float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0, c0 = a0, c1 = a0;
            const float* tr0 = Ls + (32 + i0) * LSTRIDE + 32;
            const float* tr1 = tr0 + LSTRIDE;
            for (int mb = mlo; mb < mhi; mb += 8) {  // 0, 1 or 2 blocks of 8, warp-uniform
    #pragma unroll
                for (int m = 0; m < 8; m += 2) {
                    const float2 p0 = *reinterpret_cast<const float2*>(tr0 + mb + m);
                    const float2 p1 = *reinterpret_cast<const float2*>(tr1 + mb + m);
                    const float4 l0 = ld4(Ls + (32 + mb + m) * LSTRIDE + j0), l1 = ld4(Ls + (33 + mb + m) * LSTRIDE + j0);
                    fma4(a0, p0.x, l0); fma4(a1, p1.x, l0);
                    fma4(c0, p0.y, l1); fma4(c1, p1.y, l1);
                }
            }
            a0 = make_float4(a0.x + c0.x, a0.y + c0.y, a0.z + c0.z, a0.w + c0.w);
            a1 = make_float4(a1.x + c1.x, a1.y + c1.y, a1.z + c1.z, a1.w + c1.w);
            float* part = X + 1600 + 8 * t;
            if (kh) {
                *reinterpret_cast<float4*>(part) = a0;
                *reinterpret_cast<float4*>(part + 4) = a1;
            }
            sync();
            if (!kh) {
                const float4 b0 = ld4(part), b1 = ld4(part + 4);
                float* xt = X + 512 + i0;
                xt[(j0 + 0) * 34] = a0.x + b0.x;
                xt[(j0 + 1) * 34] = a0.y + b0.y;
                xt[(j0 + 2) * 34] = a0.z + b0.z;
                xt[(j0 + 3) * 34] = a0.w + b0.w;
                xt[(j0 + 0) * 34 + 1] = a1.x + b1.x;
                xt[(j0 + 1) * 34 + 1] = a1.y + b1.y;
                xt[(j0 + 2) * 34 + 1] = a1.z + b1.z;
                xt[(j0 + 3) * 34 + 1] = a1.w + b1.w;
            }
        }
        sync();
        // E: T_[32:,:32] = -X2 T_[:32,:32]   (T_[:32,:32][m][j] = 0 for m < j). A thread takes a
        // 2x4 tile (rows 2rp, 2rp+1, columns 4cg..4cg+3) over half of the m range (threads
        // 128-255 the upper half, their partial sums handed over in X[1600 + 8t]); each warp
        // starts at the first m where its two column groups of T can be nonzero (warp-uniform),
        // and the zeros of T above the diagonal make the rest of the range exact. The 2x4 tiles
        // load a third of the shared-memory bytes per product of the 1x4 form, which bounded
        // this stage.
        {
            const int kh = tid >> 7, t = tid & 127, rp = t & 15, cg = t >> 4, i0 = 2 * rp, j0 = 4 * cg;
            const int wq = t >> 5;                                // column groups 2wq, 2wq + 1
            const int mlo = kh ? (wq > 2 ? 8 * wq : 16) : 8 * wq, mhi = 16 * kh + 16;
            float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0, c0 = a0, c1 = a0;
            for (int mb = mlo; mb < mhi; mb += 8) {               // 0, 1 or 2 blocks of 8, warp-uniform
                const float* xb = X + 512 + mb * 34 + i0;
                const float* tb = Ls + mb * LSTRIDE + j0;
    #pragma unroll
                for (int m = 0; m < 8; m += 2) {
                    const float2 x0 = *reinterpret_cast<const float2*>(xb + m * 34);
                    const float2 x1 = *reinterpret_cast<const float2*>(xb + (m + 1) * 34);
                    const float4 t0 = ld4(tb + m * LSTRIDE), t1 = ld4(tb + (m + 1) * LSTRIDE);
                    fma4(a0, x0.x, t0); fma4(a1, x0.y, t0);
                    fma4(c0, x1.x, t1); fma4(c1, x1.y, t1);
                }
            }
            a0 = make_float4(a0.x + c0.x, a0.y + c0.y, a0.z + c0.z, a0.w + c0.w);
            a1 = make_float4(a1.x + c1.x, a1.y + c1.y, a1.z + c1.z, a1.w + c1.w);
            float* part = X + 1600 + 8 * t;
            if (kh) {
                *reinterpret_cast<float4*>(part) = a0;
                *reinterpret_cast<float4*>(part + 4) = a1;
            }
            sync();
            if (!kh) {
                const float4 b0 = ld4(part), b1 = ld4(part + 4);
                *reinterpret_cast<float4*>(Ls + (32 + i0) * LSTRIDE + j0) =
                    make_float4(-(a0.x + b0.x), -(a0.y + b0.y), -(a0.z + b0.z), -(a0.w + b0.w));
                *reinterpret_cast<float4*>(Ls + (33 + i0) * LSTRIDE + j0) =
                    make_float4(-(a1.x + b1.x), -(a1.y + b1.y), -(a1.z + b1.z), -(a1.w + b1.w));
            }
        }
        sync();
    }
}

}  // namespace gdn
