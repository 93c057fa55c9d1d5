// Chunked gated-delta-rule (gated DeltaNet) prefill with a fused gated-RMSNorm
// epilogue, written for B200 (sm_100a): TMA-staged tiles, tcgen05 tensor-core
// MMAs with TMEM accumulators, and the recurrent state kept on chip.
//
// One CTA owns one (sequence, v-head) pair and walks its 64-token chunks in
// order. Per chunk n (c = in-chunk cumsum of g, L = strict-lower
// beta_i (k_i.k_j) e^{c_i-c_j}, T = (I+L)^-1):
//   P1  [Q;K] K^T            -> q.k (rows 0-63) and k.k (rows 64-127)  tcgen05, M=128
//   --  L, M = scale (q k^T) * decay  (registers), T by blocked forward
//       substitution (CUDA cores, fp32)
//   P3  W    = (T diag(beta e^c)) K                                  tcgen05, M=64, N=128
//   C12 v_new^T = v^T (T diag(beta))^T - S^T W^T                    tcgen05, M=128
//   C3  o^T  = scale e^c (S^T q^T) + v_new^T M^T  (two accumulators)  tcgen05, M=128
//   C4  dS^T = (v_new e^{c_L-c})^T K                                 tcgen05, M=128, N=128
//   --  S <- e^{c_L} S + dS (fp32 registers); o -> gated RMSNorm -> y
// Transposed forms put the 128-wide feature dimension on the MMA M axis so
// every accumulator row is one TMEM lane, which makes the state update
// thread-local; the norm epilogue re-reads o through a swizzled shared tile
// with four threads per token and 16-byte loads and stores.
//
// Precision: every operand that is not already a bf16 input (S, W, T', T'',
// v_new, M) is split into bf16 hi + lo parts, so products keep ~16 mantissa
// bits; accumulation is fp32 in TMEM; the state itself is fp32 in registers.
// Exact bf16 inputs (q, k, v) enter the MMAs unscaled; per-token factors
// (e^c, e^{c_L-c}) are applied in fp32 around them.
//
// Semantics follow the reference's torch chunked fallback
// (kernels/harness/parity_test.py:35-96) and its CUDA kernels
// (kernels/chunk_delta_cuda.cu:91-674): zero-padded tail chunk, per-chunk
// cumsum, 1/sqrt(DK) query scale applied inside, fp32 final state.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <atomic>
#include <mutex>

#include "gdn_prefill.h"
#include "sm100_ptx.cuh"

namespace gdn {

constexpr int CS = 64;         // chunk length (tokens)
constexpr int HD = 128;        // head dim (DK = DV)
constexpr int NTHREADS = 256;  // 8 warps: warps w and w+4 share TMEM lane quarter w
constexpr uint32_t TMEM_COLS = 512;

// ---- shared-memory map (bytes from a 1024-aligned base) -------------------
// bf16 tiles use the 128-byte-swizzle layout TMA writes: a tile of R rows x
// 128 columns is two 64-column "panels" of R rows x 128 B; inside a panel the
// 16-byte chunk j of row r sits at chunk position j ^ (r & 7).
constexpr uint32_t OFF_QK = 0;           // panel p: q rows 0-63 | k rows 64-127 (16 KB/panel)
constexpr uint32_t OFF_V = 32768;        // v tile  [64 tok][128 dv]  (8 KB/panel)
constexpr uint32_t OFF_Z = 49152;        // z tile  [64 tok][128 dv]
constexpr uint32_t OFF_SHI = 65536;      // S^T hi  [128 dv][128 dk]  (16 KB/panel)
constexpr uint32_t OFF_SLO = 98304;      // S^T lo
constexpr uint32_t OFF_X = 131072;       // 64 KB exchange region (two phases)
constexpr uint32_t OFF_TP_HI = OFF_X + 0;       //  T'  = T diag(beta)        [64][64]
constexpr uint32_t OFF_TP_LO = OFF_X + 8192;
constexpr uint32_t OFF_TPP_HI = OFF_X + 16384;  //  T'' = T diag(beta e^c)    [64][64]
constexpr uint32_t OFF_TPP_LO = OFF_X + 24576;
constexpr uint32_t OFF_W_HI = OFF_X + 32768;    //  W   [64 tok][128 dk]  (8 KB/panel)
constexpr uint32_t OFF_W_LO = OFF_X + 49152;
constexpr uint32_t OFF_VN = OFF_X + 0;          //  v_new^T hi       [128 dv][64 tok]
constexpr uint32_t OFF_VNP_HI = OFF_X + 16384;  //  (v_new e^{cL-c})^T hi
constexpr uint32_t OFF_VNP_LO = OFF_X + 32768;  //                     lo
constexpr uint32_t OFF_VN_LO = OFF_X + 49152;   //  v_new^T lo
constexpr uint32_t OFF_XTMP = OFF_X + 0;        //  inversion scratch [3][16][16] fp32
constexpr uint32_t OFF_L = 196608;       // L / T fp32 [64][65]; later M hi/lo
constexpr uint32_t OFF_M_HI = OFF_L;     // M = scale (q k^T) * decay, [64][64] bf16
constexpr uint32_t OFF_M_LO = OFF_L + 8192;
constexpr uint32_t OFF_OST = OFF_L;      // o staging [64 tok][128 dv] bf16 after C3 (8 KB/panel)
constexpr int LSTRIDE = 65;
constexpr uint32_t OFF_MISC = OFF_L + 64 * LSTRIDE * 4;  // 213248
constexpr uint32_t MISC_C = 0;      // c        [64] f32
constexpr uint32_t MISC_BETA = 256; // beta     [64]
constexpr uint32_t MISC_EC = 512;   // e^c      [64]
constexpr uint32_t MISC_ED = 768;   // e^{cL-c} [64]
constexpr uint32_t MISC_BAR = 2304; // 6 mbarriers
constexpr uint32_t MISC_TMEM = 2368;
constexpr uint32_t MISC_FLAG = 2372;
constexpr uint32_t MISC_BYTES = 2432;
constexpr uint32_t SMEM_BYTES = OFF_MISC + MISC_BYTES;
constexpr uint32_t SMEM_ALLOC = SMEM_BYTES + 1024;  // slack for manual 1024 alignment
static_assert(SMEM_ALLOC <= 232448, "exceeds the 227 KB per-block shared memory limit");

// TMEM columns of the accumulators (all 128 lanes).
constexpr uint32_t TM_P = 0;     // [Q;K]K^T     64 cols
constexpr uint32_t TM_V = 64;    // v_new^T      64 cols
constexpr uint32_t TM_O = 128;   // S^T q^T      64 cols
constexpr uint32_t TM_O2 = 192;  // v_new^T M^T  64 cols
constexpr uint32_t TM_S = 256;   // dS^T        128 cols
constexpr uint32_t TM_W = 384;   // W (M=64 layout: token rows in lanes 0-15 of each quarter), 128 cols

// Barrier slots.
enum { BAR_Q = 0, BAR_K = 1, BAR_V = 2, BAR_Z = 3, BAR_MMA = 4 };

constexpr uint32_t WAIT_ITERS = 1u << 22;  // bounded spin (~0.3 s with backoff)

// Debug record layout (floats) per (seq, head, chunk).
constexpr int DBG_C = 0, DBG_T = 64, DBG_W = DBG_T + 4096, DBG_VN = DBG_W + 8192,
              DBG_O = DBG_VN + 8192, DBG_SC = DBG_O + 8192, DBG_REC = DBG_SC + 16384;

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
};

// Byte offset of bf16 element (row, col) in a 128B-swizzled tile whose panels
// hold `rows` rows each.
__device__ __forceinline__ uint32_t sw_off(int row, int col, int rows) {
    return (uint32_t)((col >> 6) * rows * 128 + row * 128 + ((((col & 63) >> 3) ^ (row & 7)) << 4) +
                      ((col & 7) << 1));
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

// Write 8 consecutive fp32 values as bf16 hi (and optionally lo) parts into a
// 16-byte chunk of two tiles.
__device__ __forceinline__ void put8_split(uint32_t hi_addr, uint32_t lo_addr, const float* x,
                                           bool want_lo) {
    float h[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) h[i] = bf16r(x[i]);
    st_shared_v4(hi_addr, pack_bf16(h[0], h[1]), pack_bf16(h[2], h[3]), pack_bf16(h[4], h[5]),
                 pack_bf16(h[6], h[7]));
    if (want_lo) {
        st_shared_v4(lo_addr, pack_bf16(x[0] - h[0], x[1] - h[1]), pack_bf16(x[2] - h[2], x[3] - h[3]),
                     pack_bf16(x[4] - h[4], x[5] - h[5]), pack_bf16(x[6] - h[6], x[7] - h[7]));
    }
}

// T = (I + L)^-1 for a 64x64 strictly-lower L held in Ls (stride 65), in place.
// 16x16 diagonal blocks by forward substitution (one warp each, lane = column,
// column kept in registers); off-diagonal blocks by block rows:
// T_rs = -T_rr * sum_{m=s}^{r-1} L_rm T_ms.
__device__ __forceinline__ void invert_unit_lower(float* Ls, float* X, int tid) {
    const int warp = tid >> 5, lane = tid & 31;
    if (warp < 4 && lane < 16) {
        const int b = warp, c = lane;
        float t[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            float acc = (i == c) ? 1.f : 0.f;
#pragma unroll
            for (int j = 0; j < i; ++j) acc = fmaf(-Ls[(16 * b + i) * LSTRIDE + 16 * b + j], t[j], acc);
            t[i] = acc;
        }
        __syncwarp(0x0000ffffu);
#pragma unroll
        for (int i = 0; i < 16; ++i) Ls[(16 * b + i) * LSTRIDE + 16 * b + c] = t[i];
    }
    __syncthreads();
#pragma unroll 1
    for (int r = 1; r < 4; ++r) {
        for (int e = tid; e < r * 256; e += NTHREADS) {
            const int s = e >> 8, i = (e >> 4) & 15, c = e & 15;
            float acc = 0.f;
            for (int m = s; m < r; ++m) {
                const float* lrow = Ls + (16 * r + i) * LSTRIDE + 16 * m;
                const float* tcol = Ls + (16 * m) * LSTRIDE + 16 * s + c;
#pragma unroll
                for (int l = 0; l < 16; ++l) acc = fmaf(lrow[l], tcol[l * LSTRIDE], acc);
            }
            X[e] = acc;
        }
        __syncthreads();
        for (int e = tid; e < r * 256; e += NTHREADS) {
            const int s = e >> 8, i = (e >> 4) & 15, c = e & 15;
            const float* trow = Ls + (16 * r + i) * LSTRIDE + 16 * r;
            const float* xcol = X + s * 256 + c;
            float acc = 0.f;
#pragma unroll
            for (int l = 0; l < 16; ++l) acc = fmaf(trow[l], xcol[l * 16], acc);
            Ls[(16 * r + i) * LSTRIDE + 16 * s + c] = -acc;
        }
        __syncthreads();
    }
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
constexpr float LOG2E = 1.4426950408889634f;

__global__ void __launch_bounds__(NTHREADS, 1) gdn_prefill_kernel(const __grid_constant__ Params p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    const uint32_t sb = ptx::smem_u32(smem);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int quarter = warp & 3, half = warp >> 2;
    const int row = quarter * 32 + lane;  // TMEM lane of this thread for M=128 accumulators
    const int h = blockIdx.y;
    const int seq = blockIdx.z;
    const int hq = h / (p.HV / p.HQK);

    int t_begin, len, bcoord;
    if (p.cu_seqlens != nullptr) {
        t_begin = p.cu_seqlens[seq];
        len = p.cu_seqlens[seq + 1] - t_begin;
        bcoord = 0;
    } else {
        t_begin = 0;
        len = p.T;
        bcoord = seq;
    }
    const int NC = (len + CS - 1) / CS;
    const long long tok_base = (long long)bcoord * p.T + t_begin;  // flat token index of row 0

    float* misc = reinterpret_cast<float*>(smem + OFF_MISC);
    float* c_s = misc + MISC_C / 4;
    float* beta_s = misc + MISC_BETA / 4;
    float* ec_s = misc + MISC_EC / 4;
    float* ed_s = misc + MISC_ED / 4;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFF_MISC + MISC_FLAG);
    const uint32_t bar0 = sb + OFF_MISC + MISC_BAR;
    auto bar = [&](int i) { return bar0 + 8u * (uint32_t)i; };
    float* Ls = reinterpret_cast<float*>(smem + OFF_L);
    float* X = reinterpret_cast<float*>(smem + OFF_XTMP);

    if (tid == 0) {
        for (int i = 0; i < 5; ++i) ptx::mbar_init(bar(i), 1);
        ptx::fence_mbar_init();
        *abort_flag = 0;
        ptx::prefetch_tensormap(&p.tm_q);
        ptx::prefetch_tensormap(&p.tm_k);
        ptx::prefetch_tensormap(&p.tm_v);
        if (p.gated) ptx::prefetch_tensormap(&p.tm_z);
    }
    if (warp == 0) {
        ptx::tmem_alloc(sb + OFF_MISC + MISC_TMEM, TMEM_COLS);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + OFF_MISC + MISC_TMEM);
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;  // this warp's TMEM lane quarter

    // ---- initial state: thread (dv = row, dk in [64*half, 64*half+64)) ----
    float S[64];
    {
        const size_t sbase = ((size_t)seq * p.HV + h) * HD * HD;
#pragma unroll
        for (int j = 0; j < 64; ++j) {
            const int dk = 64 * half + j;
            S[j] = (p.s0 != nullptr) ? __ldg(p.s0 + sbase + (size_t)dk * HD + row) : 0.f;
        }
#pragma unroll
        for (int ch = 0; ch < 8; ++ch)
            put8_split(sb + OFF_SHI + sw_chunk(row, 8 * half + ch, 128),
                       sb + OFF_SLO + sw_chunk(row, 8 * half + ch, 128), S + 8 * ch, true);
    }
    // Epilogue mapping: token et = tid / 4, dv slice [32*eq, 32*eq + 32).
    const int et = tid >> 2, eq = tid & 3;
    float wgt[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) wgt[j] = p.gated ? __bfloat162float(p.w[32 * eq + j]) : 0.f;

    // ---- TMA issue helpers (thread 0) ----
    uint32_t issued[5] = {0, 0, 0, 0, 0}, consumed[5] = {0, 0, 0, 0, 0};
    auto load_q = [&](int n) {
        ++issued[BAR_Q];
        ptx::mbar_arrive_expect_tx(bar(BAR_Q), 16384);
        const int t = t_begin + n * CS;
        ptx::tma_load_4d(sb + OFF_QK + 0, &p.tm_q, bar(BAR_Q), 0, hq, t, bcoord);
        ptx::tma_load_4d(sb + OFF_QK + 16384, &p.tm_q, bar(BAR_Q), 64, hq, t, bcoord);
    };
    auto load_k = [&](int n) {
        ++issued[BAR_K];
        ptx::mbar_arrive_expect_tx(bar(BAR_K), 16384);
        const int t = t_begin + n * CS;
        ptx::tma_load_4d(sb + OFF_QK + 8192, &p.tm_k, bar(BAR_K), 0, hq, t, bcoord);
        ptx::tma_load_4d(sb + OFF_QK + 16384 + 8192, &p.tm_k, bar(BAR_K), 64, hq, t, bcoord);
    };
    auto load_v = [&](int n) {
        ++issued[BAR_V];
        ptx::mbar_arrive_expect_tx(bar(BAR_V), 16384);
        const int t = t_begin + n * CS;
        ptx::tma_load_4d(sb + OFF_V + 0, &p.tm_v, bar(BAR_V), 0, h, t, bcoord);
        ptx::tma_load_4d(sb + OFF_V + 8192, &p.tm_v, bar(BAR_V), 64, h, t, bcoord);
    };
    auto load_z = [&](int n) {
        ++issued[BAR_Z];
        ptx::mbar_arrive_expect_tx(bar(BAR_Z), 16384);
        const int t = t_begin + n * CS;
        ptx::tma_load_4d(sb + OFF_Z + 0, &p.tm_z, bar(BAR_Z), 0, h, t, bcoord);
        ptx::tma_load_4d(sb + OFF_Z + 8192, &p.tm_z, bar(BAR_Z), 64, h, t, bcoord);
    };

    // Every wait is bounded; a timeout records status bit 0 and stops the CTA.
    // issued[] / consumed[] count barrier completions so the exit path can
    // drain whatever is still in flight (thread 0 issues every TMA and MMA).
    auto fail = [&]() {
        *abort_flag = 1;
        if (p.status) atomicOr(p.status, 1u);
    };
    auto wait_bar = [&](int i, uint32_t parity) {
        if (ptx::mbar_wait(bar(i), parity, WAIT_ITERS)) ++consumed[i];
        else fail();
    };
    auto wait_mma = [&]() {
        wait_bar(BAR_MMA, consumed[BAR_MMA] & 1u);
        ptx::tc_fence_after();
    };

    if (tid == 0 && NC > 0) {
        load_q(0);
        load_k(0);
        load_v(0);
        if (p.gated) load_z(0);
    }
    // Gates of the next chunk are prefetched into warp 0's registers (lane l: tokens 2l, 2l+1).
    float gn0 = 0.f, gn1 = 0.f, bn0 = 0.f, bn1 = 0.f;
    auto load_gates = [&](int n) {
        const int valid = min(CS, len - n * CS);
        const long long t0 = tok_base + (long long)n * CS;
        gn0 = gn1 = bn0 = bn1 = 0.f;
        if (2 * lane < valid) {
            gn0 = __ldg(p.g + (size_t)(t0 + 2 * lane) * p.HV + h);
            bn0 = __ldg(p.beta + (size_t)(t0 + 2 * lane) * p.HV + h);
        }
        if (2 * lane + 1 < valid) {
            gn1 = __ldg(p.g + (size_t)(t0 + 2 * lane + 1) * p.HV + h);
            bn1 = __ldg(p.beta + (size_t)(t0 + 2 * lane + 1) * p.HV + h);
        }
    };
    if (warp == 0 && NC > 0) load_gates(0);
    ptx::fence_proxy_async_smem();  // S tiles written by all threads
    __syncthreads();

    // Instruction descriptors.
    constexpr uint32_t ID_P = ptx::idesc_bf16(128, 64, 0, 0, 0);    // [Q;K] K^T
    constexpr uint32_t ID_W = ptx::idesc_bf16(64, 128, 0, 1, 0);    // T'' K        (B MN-major)
    constexpr uint32_t ID_U = ptx::idesc_bf16(128, 64, 1, 0, 0);    // v^T T'^T     (A MN-major)
    constexpr uint32_t ID_WS = ptx::idesc_bf16(128, 64, 0, 0, 1);   // -S^T W^T
    constexpr uint32_t ID_O = ptx::idesc_bf16(128, 64, 0, 0, 0);    // S^T q^T, v_new^T M^T
    constexpr uint32_t ID_S = ptx::idesc_bf16(128, 128, 0, 1, 0);   // v_new'^T K   (B MN-major)

    for (int n = 0; n < NC; ++n) {
        if (*abort_flag) break;
        const int valid = min(CS, len - n * CS);
        const long long tok0 = tok_base + (long long)n * CS;
        const uint32_t ph = (uint32_t)(n & 1);

        // ---- gates: in-chunk inclusive cumsum of g (warp scan), decay factors ----
        if (warp == 0) {
            const float g0 = gn0, g1 = gn1, b0 = bn0, b1 = bn1;
            if (n + 1 < NC) load_gates(n + 1);  // overlaps the rest of this chunk
            float s = g0 + g1;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const float t = __shfl_up_sync(0xffffffffu, s, off);
                if (lane >= off) s += t;
            }
            const float c1 = s, c0 = s - g1;
            const float cL = __shfl_sync(0xffffffffu, c1, 31);
            c_s[2 * lane] = c0;
            c_s[2 * lane + 1] = c1;
            beta_s[2 * lane] = b0;
            beta_s[2 * lane + 1] = b1;
            ec_s[2 * lane] = ex2f(c0 * LOG2E);
            ec_s[2 * lane + 1] = ex2f(c1 * LOG2E);
            ed_s[2 * lane] = ex2f((cL - c0) * LOG2E);
            ed_s[2 * lane + 1] = ex2f((cL - c1) * LOG2E);
        }

        // ---- P1: [Q;K] K^T ----
        wait_bar(BAR_Q, ph);
        wait_bar(BAR_K, ph);
        if (tid == 0) {
            ptx::tc_fence_after();
#pragma unroll
            for (int s = 0; s < 8; ++s) {
                const uint32_t koff = (uint32_t)(s >> 2) * 16384u + (uint32_t)(s & 3) * 32u;
                const uint64_t a = ptx::sw128_desc(sb + OFF_QK + koff, 16, 1024);
                const uint64_t b = ptx::sw128_desc(sb + OFF_QK + 8192 + koff, 16, 1024);
                ptx::mma_bf16(tmem + TM_P, a, b, ID_P, s > 0);
            }
            ptx::mma_commit(bar(BAR_MMA));
            ++issued[BAR_MMA];
        }
        __syncthreads();  // c_s / beta_s visible
        wait_mma();
        {
            float v[32];
            ptx::tmem_ld32(tmem + lane_addr + TM_P + 32 * half, v);
            ptx::tmem_wait_ld();
            // rows 0-63 (q.k) stay in TMEM until M is formed after C12
            if (row >= CS) {  // L row i: beta_i k_i.k_j e^{c_i - c_j}, j < i
                const int i = row - CS;
                const float ci = c_s[i], bi = beta_s[i];
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) {
                    const int j = 32 * half + jj;
                    Ls[i * LSTRIDE + j] = (j < i) ? bi * v[jj] * ex2f((ci - c_s[j]) * LOG2E) : 0.f;
                }
            }
        }
        ptx::tc_fence_before();
        __syncthreads();

        // ---- T = (I + L)^-1 (fp32, CUDA cores) ----
        invert_unit_lower(Ls, X, tid);
        if (p.dbg) {
            float* rec = p.dbg + (((size_t)seq * p.HV + h) * p.max_nc + n) * DBG_REC;
            for (int e = tid; e < CS * CS; e += NTHREADS) rec[DBG_T + e] = Ls[(e >> 6) * LSTRIDE + (e & 63)];
            if (tid < CS) rec[DBG_C + tid] = c_s[tid];
        }
        // T' = T diag(beta), T'' = T diag(beta e^c): hi/lo bf16 tiles [64][64]
        {
            const int i = tid >> 2, jb = tid & 3;
            float tp[16], tpp[16];
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) {
                const int j = 16 * jb + jj;
                const float t = Ls[i * LSTRIDE + j];
                tp[jj] = t * beta_s[j];
                tpp[jj] = tp[jj] * ec_s[j];
            }
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const uint32_t co = sw_chunk(i, 2 * jb + hh, 64);
                put8_split(sb + OFF_TP_HI + co, sb + OFF_TP_LO + co, tp + 8 * hh, true);
                put8_split(sb + OFF_TPP_HI + co, sb + OFF_TPP_LO + co, tpp + 8 * hh, true);
            }
        }
        ptx::fence_proxy_async_smem();
        __syncthreads();

        // ---- P3: W = T'' K (hi + lo), M = 64 tokens x N = 128 dk ----
        if (tid == 0) {
            ptx::tc_fence_after();
#pragma unroll
            for (int part = 0; part < 2; ++part) {
                const uint32_t tpp = part ? OFF_TPP_LO : OFF_TPP_HI;
#pragma unroll
                for (int s = 0; s < 4; ++s) {
                    const uint64_t a = ptx::sw128_desc(sb + tpp + s * 32, 16, 1024);
                    const uint64_t b = ptx::sw128_desc(sb + OFF_QK + 8192 + s * 2048, 16384, 1024);
                    ptx::mma_bf16(tmem + TM_W, a, b, ID_W, (part | s) > 0);
                }
            }
            ptx::mma_commit(bar(BAR_MMA));
            ++issued[BAR_MMA];
        }
        wait_mma();
        {   // M=64 accumulator: token 16*quarter + lane (lanes 0-15), dk 64*half .. +63
#pragma unroll
            for (int c2 = 0; c2 < 2; ++c2) {
                float v[32];
                ptx::tmem_ld32(tmem + lane_addr + TM_W + 64 * half + 32 * c2, v);
                ptx::tmem_wait_ld();
                if (lane < 16) {
                    const int tok = 16 * quarter + lane;
#pragma unroll
                    for (int ch = 0; ch < 4; ++ch) {
                        const uint32_t co = sw_chunk(tok, 8 * half + 4 * c2 + ch, 64);
                        put8_split(sb + OFF_W_HI + co, sb + OFF_W_LO + co, v + 8 * ch, true);
                    }
                    if (p.dbg) {
                        float* rec = p.dbg + (((size_t)seq * p.HV + h) * p.max_nc + n) * DBG_REC;
#pragma unroll
                        for (int jj = 0; jj < 32; ++jj) rec[DBG_W + tok * HD + 64 * half + 32 * c2 + jj] = v[jj];
                    }
                }
            }
        }
        ptx::tc_fence_before();
        ptx::fence_proxy_async_smem();
        __syncthreads();
        if (*abort_flag) break;

        // ---- C12: v_new^T = v^T T'^T - S^T W^T ----
        wait_bar(BAR_V, ph);
        if (tid == 0) {
            ptx::tc_fence_after();
            bool first = true;
#pragma unroll
            for (int part = 0; part < 2; ++part) {
                const uint32_t tp = part ? OFF_TP_LO : OFF_TP_HI;
#pragma unroll
                for (int s = 0; s < 4; ++s) {
                    const uint64_t a = ptx::sw128_desc(sb + OFF_V + s * 2048, 8192, 1024);
                    const uint64_t b = ptx::sw128_desc(sb + tp + s * 32, 16, 1024);
                    ptx::mma_bf16(tmem + TM_V, a, b, ID_U, first ? 0u : 1u);
                    first = false;
                }
            }
            // (S_hi, W_hi), (S_lo, W_hi), (S_hi, W_lo)
#pragma unroll
            for (int term = 0; term < 3; ++term) {
                const uint32_t sa = (term == 1) ? OFF_SLO : OFF_SHI;
                const uint32_t wb = (term == 2) ? OFF_W_LO : OFF_W_HI;
#pragma unroll
                for (int s = 0; s < 8; ++s) {
                    const uint64_t a =
                        ptx::sw128_desc(sb + sa + (s >> 2) * 16384 + (s & 3) * 32, 16, 1024);
                    const uint64_t b = ptx::sw128_desc(sb + wb + (s >> 2) * 8192 + (s & 3) * 32, 16, 1024);
                    ptx::mma_bf16(tmem + TM_V, a, b, ID_WS, 1u);
                }
            }
            ptx::mma_commit(bar(BAR_MMA));
            ++issued[BAR_MMA];
        }
        wait_mma();
        if (tid == 0 && n + 1 < NC) load_v(n + 1);  // v tile consumed
        {
            float v[32];
            ptx::tmem_ld32(tmem + lane_addr + TM_V + 32 * half, v);
            ptx::tmem_wait_ld();
            const int dv = row;
            float vp[32];
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) vp[jj] = v[jj] * ed_s[32 * half + jj];
#pragma unroll
            for (int ch = 0; ch < 4; ++ch) {
                const uint32_t co = sw_chunk(dv, 4 * half + ch, 128);
                put8_split(sb + OFF_VN + co, sb + OFF_VN_LO + co, v + 8 * ch, true);
                put8_split(sb + OFF_VNP_HI + co, sb + OFF_VNP_LO + co, vp + 8 * ch, true);
            }
            if (p.dbg) {
                float* rec = p.dbg + (((size_t)seq * p.HV + h) * p.max_nc + n) * DBG_REC;
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) rec[DBG_VN + (32 * half + jj) * HD + dv] = v[jj];
            }
        }
        {   // M row i: scale * (q_i.k_j) * e^{c_i - c_j} for j <= i, hi/lo, from the P1 accumulator
            float v[32];
            ptx::tmem_ld32(tmem + lane_addr + TM_P + 32 * half, v);
            ptx::tmem_wait_ld();
            if (row < CS) {
                const int i = row;
                const float ci = c_s[i];
                float m[32];
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) {
                    const int j = 32 * half + jj;
                    m[jj] = (j <= i) ? v[jj] * p.scale * ex2f((ci - c_s[j]) * LOG2E) : 0.f;
                }
#pragma unroll
                for (int ch = 0; ch < 4; ++ch) {
                    const uint32_t co = sw_chunk(i, 4 * half + ch, 64);
                    put8_split(sb + OFF_M_HI + co, sb + OFF_M_LO + co, m + 8 * ch, true);
                }
            }
        }
        ptx::tc_fence_before();
        ptx::fence_proxy_async_smem();
        __syncthreads();
        if (*abort_flag) break;

        // ---- C3: o1^T = S^T q^T, o2^T = v_new^T M^T ; C4: dS^T = v_new'^T K ----
        if (tid == 0) {
            ptx::tc_fence_after();
#pragma unroll
            for (int part = 0; part < 2; ++part) {
                const uint32_t sa = part ? OFF_SLO : OFF_SHI;
#pragma unroll
                for (int s = 0; s < 8; ++s) {
                    const uint64_t a =
                        ptx::sw128_desc(sb + sa + (s >> 2) * 16384 + (s & 3) * 32, 16, 1024);
                    const uint64_t b = ptx::sw128_desc(sb + OFF_QK + (s >> 2) * 16384 + (s & 3) * 32, 16, 1024);
                    ptx::mma_bf16(tmem + TM_O, a, b, ID_O, (part | s) > 0);
                }
            }
            // (VN_hi, M_hi), (VN_lo, M_hi), (VN_hi, M_lo)
#pragma unroll
            for (int term = 0; term < 3; ++term) {
                const uint32_t va = (term == 1) ? OFF_VN_LO : OFF_VN;
                const uint32_t mb = (term == 2) ? OFF_M_LO : OFF_M_HI;
#pragma unroll
                for (int s = 0; s < 4; ++s) {
                    const uint64_t a = ptx::sw128_desc(sb + va + s * 32, 16, 1024);
                    const uint64_t b = ptx::sw128_desc(sb + mb + s * 32, 16, 1024);
                    ptx::mma_bf16(tmem + TM_O2, a, b, ID_O, (term | s) > 0);
                }
            }
#pragma unroll
            for (int part = 0; part < 2; ++part) {
                const uint32_t va = part ? OFF_VNP_LO : OFF_VNP_HI;
#pragma unroll
                for (int s = 0; s < 4; ++s) {
                    const uint64_t a = ptx::sw128_desc(sb + va + s * 32, 16, 1024);
                    const uint64_t b = ptx::sw128_desc(sb + OFF_QK + 8192 + s * 2048, 16384, 1024);
                    ptx::mma_bf16(tmem + TM_S, a, b, ID_S, (part | s) > 0);
                }
            }
            ptx::mma_commit(bar(BAR_MMA));
            ++issued[BAR_MMA];
        }
        wait_mma();
        if (tid == 0 && n + 1 < NC) {  // q and k tiles consumed
            load_q(n + 1);
            load_k(n + 1);
        }

        // ---- state update: S <- e^{cL} S + dS ----
        {
            const float gam = ec_s[CS - 1];
            if (p.dbg) {
                float* rec = p.dbg + (((size_t)seq * p.HV + h) * p.max_nc + n) * DBG_REC;
#pragma unroll
                for (int j = 0; j < 64; ++j) rec[DBG_SC + (64 * half + j) * HD + row] = S[j];
            }
#pragma unroll
            for (int c2 = 0; c2 < 2; ++c2) {
                float v[32];
                ptx::tmem_ld32(tmem + lane_addr + TM_S + 64 * half + 32 * c2, v);
                ptx::tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 32; ++j) S[32 * c2 + j] = fmaf(gam, S[32 * c2 + j], v[j]);
            }
#pragma unroll
            for (int ch = 0; ch < 8; ++ch)
                put8_split(sb + OFF_SHI + sw_chunk(row, 8 * half + ch, 128),
                           sb + OFF_SLO + sw_chunk(row, 8 * half + ch, 128), S + 8 * ch, true);
        }

        // ---- o = scale e^c o1 + o2, rounded to bf16, staged [tok][dv] (M tiles are dead) ----
        {
            float v[32], v2[32];
            ptx::tmem_ld32(tmem + lane_addr + TM_O + 32 * half, v);
            ptx::tmem_ld32(tmem + lane_addr + TM_O2 + 32 * half, v2);
            ptx::tmem_wait_ld();
            const int dv = row;
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) v[jj] = fmaf(p.scale * ec_s[32 * half + jj], v[jj], v2[jj]);
            if (p.dbg) {
                float* rec = p.dbg + (((size_t)seq * p.HV + h) * p.max_nc + n) * DBG_REC;
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) rec[DBG_O + (32 * half + jj) * HD + dv] = v[jj];
            }
            __nv_bfloat16* ot = reinterpret_cast<__nv_bfloat16*>(smem + OFF_OST);
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) ot[sw_off(32 * half + jj, dv, 64) >> 1] = __float2bfloat16_rn(v[jj]);
        }
        ptx::tc_fence_before();
        ptx::fence_proxy_async_smem();  // S tiles
        __syncthreads();

        // ---- epilogue: 4 threads per token, 32 dv each, 16-byte accesses ----
        {
            float o[32];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                uint32_t w4[4];
                ld_shared_v4(sb + OFF_OST + sw_chunk(et, 4 * eq + c, 64), w4[0], w4[1], w4[2], w4[3]);
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const __nv_bfloat162 b2 = *reinterpret_cast<const __nv_bfloat162*>(&w4[u]);
                    o[8 * c + 2 * u] = __bfloat162float(b2.x);
                    o[8 * c + 2 * u + 1] = __bfloat162float(b2.y);
                }
            }
            uint32_t outw[16];
            if (!p.gated) {
#pragma unroll
                for (int j = 0; j < 16; ++j) outw[j] = pack_bf16(o[2 * j], o[2 * j + 1]);
            } else {
                float ss = 0.f;
#pragma unroll
                for (int j = 0; j < 32; ++j) ss = fmaf(o[j], o[j], ss);
                ss += __shfl_xor_sync(0xffffffffu, ss, 1);
                ss += __shfl_xor_sync(0xffffffffu, ss, 2);
                const float rstd = rsqrtf(ss * (1.f / (float)HD) + p.eps);
                wait_bar(BAR_Z, ph);
                float y[32];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    uint32_t w4[4];
                    ld_shared_v4(sb + OFF_Z + sw_chunk(et, 4 * eq + c, 64), w4[0], w4[1], w4[2], w4[3]);
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const __nv_bfloat162 b2 = *reinterpret_cast<const __nv_bfloat162*>(&w4[u]);
                        const float zz[2] = {__bfloat162float(b2.x), __bfloat162float(b2.y)};
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            const int j = 8 * c + 2 * u + e;
                            const float nb = bf16r(o[j] * rstd);
                            const float sg = zz[e] * rcpf(1.f + ex2f(-zz[e] * LOG2E));
                            y[j] = (wgt[j] * nb) * sg;
                        }
                    }
                }
#pragma unroll
                for (int j = 0; j < 16; ++j) outw[j] = pack_bf16(y[2 * j], y[2 * j + 1]);
            }
            if (et < valid) {
                uint4* dst = reinterpret_cast<uint4*>(p.out + (size_t)(tok0 + et) * p.HV * HD + (size_t)h * HD +
                                                      32 * eq);
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    dst[c] = make_uint4(outw[4 * c], outw[4 * c + 1], outw[4 * c + 2], outw[4 * c + 3]);
            }
        }
        __syncthreads();
        if (tid == 0 && p.gated && n + 1 < NC) {
            ptx::fence_proxy_async_smem();
            load_z(n + 1);  // z tile consumed
        }
    }

    // ---- final state ----
    if (!*abort_flag) {
        const size_t sbase = ((size_t)seq * p.HV + h) * HD * HD;
#pragma unroll
        for (int j = 0; j < 64; ++j) {
            const int dk = 64 * half + j;
            p.sf[sbase + (size_t)dk * HD + row] = S[j];
        }
    }
    // Abort path: wait (bounded) for this CTA's own TMA copies and MMAs still
    // in flight before its shared memory and TMEM are released.
    if (*abort_flag && tid == 0) {
        for (int i = 0; i < 5; ++i)
            while (consumed[i] < issued[i]) {
                ptx::mbar_wait(bar(i), consumed[i] & 1u, WAIT_ITERS);
                ++consumed[i];
            }
    }
    ptx::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem, TMEM_COLS);
    }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
    static std::once_flag once;
    static EncodeTiledFn fn = nullptr;
    std::call_once(once, []() {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult qres;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &qres) ==
                cudaSuccess &&
            qres == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    });
    return fn;
}

// 4-D bf16 tensor map over [B][T][H][128] (inner -> outer: dim, head, token, batch),
// box 64 x 1 x 64 x 1 with 128-byte swizzle; out-of-bounds rows read as zero.
static bool make_map(CUtensorMap* m, const void* base, int H, int T, int B) {
    EncodeTiledFn enc = get_encode_fn();
    if (!enc) return false;
    cuuint64_t dims[4] = {(cuuint64_t)HD, (cuuint64_t)H, (cuuint64_t)T, (cuuint64_t)B};
    cuuint64_t strides[3] = {(cuuint64_t)HD * 2, (cuuint64_t)H * HD * 2, (cuuint64_t)T * H * HD * 2};
    cuuint32_t box[4] = {64, 1, 64, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides,
                     box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static cudaError_t ensure_smem_attr() {
    static std::atomic<uint64_t> done_mask{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = (dev < 64) ? (1ull << dev) : 0;
    if (bit && (done_mask.load(std::memory_order_acquire) & bit)) return cudaSuccess;
    e = cudaFuncSetAttribute(gdn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)SMEM_ALLOC);
    if (e == cudaSuccess && bit) done_mask.fetch_or(bit, std::memory_order_acq_rel);
    return e;
}

constexpr size_t WS_HEADER = 256;

struct Launch {
    const void *q, *k, *v;
    const float *g, *beta;
    const void *z, *w;
    float eps;
    void* out;
    const float* s0;
    float* sf;
    const int* cu;
    int nseq, T, HV, HQK, DK, DV, chunk, B;
    int max_nc;
    void* ws;
    size_t ws_bytes;
    float* dbg;
    cudaStream_t stream;
};

static cudaError_t launch(const Launch& L) {
    if (L.DK != HD || L.DV != HD || L.chunk != CS) return cudaErrorInvalidValue;
    if (L.HQK <= 0 || L.HV <= 0 || L.HV % L.HQK != 0) return cudaErrorInvalidValue;
    if (L.T < 0 || L.nseq < 0 || L.HV > 65535 || L.nseq > 65535) return cudaErrorInvalidValue;
    if (!L.q || !L.k || !L.v || !L.g || !L.beta || !L.out || !L.sf || !L.ws)
        return cudaErrorInvalidValue;
    if (L.ws_bytes < WS_HEADER) return cudaErrorInvalidValue;
    const bool gated = (L.z != nullptr) || (L.w != nullptr);
    if (gated && (!L.z || !L.w)) return cudaErrorInvalidValue;
    if (!aligned16(L.q) || !aligned16(L.k) || !aligned16(L.v) || (gated && !aligned16(L.z)) ||
        !aligned16(L.ws) || !aligned16(L.out))
        return cudaErrorInvalidValue;
    if (L.nseq == 0 || L.HV == 0) return cudaSuccess;

    Params p;
    memset(&p, 0, sizeof(p));
    const int Bmap = L.cu ? 1 : L.B;
    const int Tmap = L.T > 0 ? L.T : 1;
    if (!make_map(&p.tm_q, L.q, L.HQK, Tmap, Bmap) || !make_map(&p.tm_k, L.k, L.HQK, Tmap, Bmap) ||
        !make_map(&p.tm_v, L.v, L.HV, Tmap, Bmap))
        return cudaErrorInvalidValue;
    if (gated) {
        if (!make_map(&p.tm_z, L.z, L.HV, Tmap, Bmap)) return cudaErrorInvalidValue;
    } else {
        p.tm_z = p.tm_v;
    }
    p.g = L.g;
    p.beta = L.beta;
    p.w = static_cast<const __nv_bfloat16*>(L.w);
    p.s0 = L.s0;
    p.sf = L.sf;
    p.out = static_cast<__nv_bfloat16*>(L.out);
    p.cu_seqlens = L.cu;
    p.status = static_cast<unsigned int*>(L.ws);
    p.dbg = L.dbg;
    p.T = L.T;
    p.HV = L.HV;
    p.HQK = L.HQK;
    p.max_nc = L.max_nc;
    p.scale = 1.0f / sqrtf((float)L.DK);
    p.eps = L.eps;
    p.gated = gated ? 1 : 0;

    cudaError_t e = ensure_smem_attr();
    if (e != cudaSuccess) return e;
    dim3 grid(1, L.HV, L.nseq);
    gdn_prefill_kernel<<<grid, NTHREADS, SMEM_ALLOC, L.stream>>>(p);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Scratch for callers that cannot allocate device memory (see
// deltanet_chunk_prefill_gated_noalloc). A file-scope device array that every
// GPU loading this library holds until exit; its host-side name is only a
// stand-in, so the device address is looked up once per device with
// cudaGetSymbolAddress while that device is current.
constexpr size_t NOALLOC_SCRATCH_BYTES = 256;  // maximum scratch the no-alloc entry can serve
static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];
constexpr int NOALLOC_MAX_DEVICES = 64;

static cudaError_t noalloc_scratch(void** out) {
    static std::mutex mu;
    static void* addr[NOALLOC_MAX_DEVICES] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= NOALLOC_MAX_DEVICES) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(mu);
    if (addr[dev] == nullptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        addr[dev] = p;
    }
    *out = addr[dev];
    return cudaSuccess;
}

static size_t debug_bytes(int B, int T, int HV) {
    const size_t nc = (size_t)((T + CS - 1) / CS);
    return (size_t)B * HV * nc * DBG_REC * sizeof(float);
}

}  // namespace gdn

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
extern "C" {

size_t deltanet_prefill_workspace_size(int B, int T, int HV, int DK, int DV, int chunk_size) {
    (void)B; (void)T; (void)HV; (void)DK; (void)DV; (void)chunk_size;
    return gdn::WS_HEADER;
}

size_t deltanet_prefill_debug_workspace_size(int B, int T, int HV, int DK, int DV, int chunk_size) {
    (void)DK; (void)DV; (void)chunk_size;
    return gdn::WS_HEADER + gdn::debug_bytes(B, T, HV);
}

cudaError_t deltanet_chunk_prefill(const void* q, const void* k, const void* v, const float* g,
                                   const float* beta, void* o, const float* initial_state,
                                   float* final_state, int B, int T, int HV, int HQK, int DK, int DV,
                                   int chunk_size, void* workspace, size_t workspace_bytes,
                                   cudaStream_t stream, int dump_debug) {
    gdn::Launch L;
    memset(&L, 0, sizeof(L));
    L.q = q; L.k = k; L.v = v; L.g = g; L.beta = beta; L.out = o;
    L.s0 = initial_state; L.sf = final_state;
    L.nseq = B; L.B = B; L.T = T; L.HV = HV; L.HQK = HQK; L.DK = DK; L.DV = DV; L.chunk = chunk_size;
    L.max_nc = (T + gdn::CS - 1) / gdn::CS;
    L.ws = workspace; L.ws_bytes = workspace_bytes; L.stream = stream;
    if (dump_debug) {
        if (workspace_bytes < deltanet_prefill_debug_workspace_size(B, T, HV, DK, DV, chunk_size))
            return cudaErrorInvalidValue;
        L.dbg = reinterpret_cast<float*>(static_cast<char*>(workspace) + gdn::WS_HEADER);
    }
    return gdn::launch(L);
}

size_t deltanet_tcop_prefill_workspace_size(int B, int T, int HV, int DK, int DV, int chunk_size) {
    return deltanet_prefill_workspace_size(B, T, HV, DK, DV, chunk_size);
}

cudaError_t deltanet_tcop_chunk_prefill(const void* q, const void* k, const void* v, const float* g,
                                        const float* beta, void* o, const float* initial_state,
                                        float* final_state, int B, int T, int HV, int HQK, int DK,
                                        int DV, int chunk_size, void* workspace,
                                        size_t workspace_bytes, cudaStream_t stream, int dump_debug) {
    return deltanet_chunk_prefill(q, k, v, g, beta, o, initial_state, final_state, B, T, HV, HQK, DK,
                                  DV, chunk_size, workspace, workspace_bytes, stream, dump_debug);
}

cudaError_t deltanet_chunk_prefill_gated(const void* q, const void* k, const void* v, const float* g,
                                         const float* beta, const void* z, const void* norm_w,
                                         float eps, void* y, const float* initial_state,
                                         float* final_state, int B, int T, int HV, int HQK, int DK,
                                         int DV, int chunk_size, void* workspace,
                                         size_t workspace_bytes, cudaStream_t stream) {
    if (!z || !norm_w) return cudaErrorInvalidValue;
    gdn::Launch L;
    memset(&L, 0, sizeof(L));
    L.q = q; L.k = k; L.v = v; L.g = g; L.beta = beta; L.z = z; L.w = norm_w; L.eps = eps; L.out = y;
    L.s0 = initial_state; L.sf = final_state;
    L.nseq = B; L.B = B; L.T = T; L.HV = HV; L.HQK = HQK; L.DK = DK; L.DV = DV; L.chunk = chunk_size;
    L.max_nc = (T + gdn::CS - 1) / gdn::CS;
    L.ws = workspace; L.ws_bytes = workspace_bytes; L.stream = stream;
    return gdn::launch(L);
}

cudaError_t deltanet_chunk_prefill_varlen(const void* q, const void* k, const void* v, const float* g,
                                          const float* beta, const void* z, const void* norm_w,
                                          float eps, void* out, const float* initial_states,
                                          float* final_states, const int* cu_seqlens, int N, int T,
                                          int HV, int HQK, int DK, int DV, int chunk_size,
                                          void* workspace, size_t workspace_bytes,
                                          cudaStream_t stream) {
    if (!cu_seqlens || N < 0) return cudaErrorInvalidValue;
    if ((z == nullptr) != (norm_w == nullptr)) return cudaErrorInvalidValue;
    gdn::Launch L;
    memset(&L, 0, sizeof(L));
    L.q = q; L.k = k; L.v = v; L.g = g; L.beta = beta; L.z = z; L.w = norm_w; L.eps = eps; L.out = out;
    L.s0 = initial_states; L.sf = final_states; L.cu = cu_seqlens;
    L.nseq = N; L.B = 1; L.T = T; L.HV = HV; L.HQK = HQK; L.DK = DK; L.DV = DV; L.chunk = chunk_size;
    L.max_nc = (T + gdn::CS - 1) / gdn::CS;
    L.ws = workspace; L.ws_bytes = workspace_bytes; L.stream = stream;
    return gdn::launch(L);
}

// Same computation as deltanet_chunk_prefill_gated, with its scratch (the
// status word the bounded waits report to) taken from a static device array
// instead of a caller-provided workspace, so the call performs no device
// allocation at all (no cudaMalloc/cudaFree, no library allocator).
// The first call on each device looks the array's address up, so make that
// first call before any stream capture. Every call shares the one array:
// calls whose kernels overlap on the GPU (concurrent streams) race on it; the
// status word is cleared on `stream` before each launch.
cudaError_t deltanet_chunk_prefill_gated_noalloc(const void* q, const void* k, const void* v,
                                                 const float* g, const float* beta, const void* z,
                                                 const void* norm_w, float eps, void* y,
                                                 const float* initial_state, float* final_state,
                                                 int B, int T, int HV, int HQK, int DK, int DV,
                                                 int chunk_size, cudaStream_t stream) {
    const size_t need = deltanet_prefill_workspace_size(B, T, HV, DK, DV, chunk_size);
    if (need > gdn::NOALLOC_SCRATCH_BYTES) return cudaErrorInvalidValue;  // beyond the static maximum
    void* ws = nullptr;
    cudaError_t e = gdn::noalloc_scratch(&ws);
    if (e != cudaSuccess) return e;
    e = cudaMemsetAsync(ws, 0, need, stream);  // the status word must start at zero
    if (e != cudaSuccess) return e;
    return deltanet_chunk_prefill_gated(q, k, v, g, beta, z, norm_w, eps, y, initial_state, final_state, B, T,
                                        HV, HQK, DK, DV, chunk_size, ws, gdn::NOALLOC_SCRATCH_BYTES, stream);
}

cudaError_t deltanet_read_status(void* workspace, int* status_host, int clear, cudaStream_t stream) {
    if (!workspace || !status_host) return cudaErrorInvalidValue;
    unsigned int s = 0;
    cudaError_t e = cudaMemcpyAsync(&s, workspace, sizeof(s), cudaMemcpyDeviceToHost, stream);
    if (e != cudaSuccess) return e;
    e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return e;
    *status_host = (int)s;
    if (clear) e = cudaMemsetAsync(workspace, 0, sizeof(s), stream);
    return e;
}

const char* gdn_b200_version(void) { return "gdn_b200 0.1 (sm_100a, tcgen05 fused prefill)"; }

}  // extern "C"
