// Cluster-split variant of the chunked gated-delta-rule prefill for small
// batches (few (sequence, v-head) units relative to the 148 SMs).
//
// Each (sequence, v-head) runs on a cluster of 1 + NP CTAs:
//   * rank 0, the chain CTA, owns the recurrent state and runs only the
//     state-dependent steps of every chunk: C12 (v_new), C3/C4 (output and
//     state increment), the state update and the gated-RMSNorm epilogue;
//   * ranks 1..NP, the prep CTAs, run the state-independent chunk math for
//     chunks n = rank-1, rank-1+NP, ...: gates, P1 ([Q;K]K^T), L and M, the
//     triangular inverse, T' and T'', P3 (W), and ship T' / W / M / decay
//     factors into the chain CTA's slot buffer with one shared-to-shared bulk
//     copy per chunk (completing on the chain's mbarrier; no multicast).
// Prep and chain of different chunks overlap, so the chain's period per
// chunk is its own work only. The math, precision scheme and operand
// layouts are those of gdn_prefill_kernel (gdn_prefill.cu).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "gdn_common.cuh"
#include "gdn_prefill.h"
#include "sm100_ptx.cuh"

namespace gdn {
namespace split {

constexpr int NTHREADS = 256;
constexpr int NP = 2;  // prep CTAs per cluster

// ---- slot layout (identical in the prep CTA's staging and the chain CTA's slots)
constexpr uint32_t SL_TP = 0;        // [T'_hi; T'_lo] 128 rows x 64 cols bf16 (K-major, stacked along N)
constexpr uint32_t SL_W = 16384;     // W^T hi, lo: [128 dk][64 tok] bf16 MN-major tiles, 16 KB apart
constexpr uint32_t SL_M = 49152;     // M hi, lo: [64][64] bf16, 8 KB apart
constexpr uint32_t SL_EC = 65536;    // e^c      [64] f32
constexpr uint32_t SL_ED = 65792;    // e^{cL-c} [64] f32
constexpr uint32_t SL_BYTES = 66048; // bytes shipped per chunk
constexpr uint32_t SLOT = 66560;     // slot stride (1024-aligned)

// ---- chain CTA shared memory
constexpr uint32_t C_QK = 0;          // q rows 0-63 | k rows 64-127 (16 KB/panel)
constexpr uint32_t C_V = 32768;
constexpr uint32_t C_Z = 49152;
constexpr uint32_t C_SLOT = 65536;    // NP slots
constexpr uint32_t C_OST = C_SLOT + NP * SLOT;   // o staging [64 tok][128 dv] bf16 (8 KB/panel)
constexpr uint32_t C_MISC = C_OST + 16384;
// ---- prep CTA shared memory
constexpr uint32_t P_QK = 0;
constexpr uint32_t P_L = 32768;                  // L / T fp32 [64][68]
constexpr uint32_t P_TPP = 50176;                // T'' hi, lo [64][64] bf16
constexpr uint32_t P_STG = 66560;                // 2 staging slots
constexpr uint32_t P_MISC = P_STG + 2 * SLOT;
// ---- misc (both roles)
constexpr uint32_t M_C = 0, M_BETA = 256, M_W = 512, M_BAR = 1024, M_TMEM = 1152, M_FLAG = 1156, M_BYTES = 1280;
constexpr uint32_t SMEM_BYTES = (C_MISC > P_MISC ? C_MISC : P_MISC) + M_BYTES;
constexpr uint32_t SMEM_ALLOC = SMEM_BYTES + 1024;
static_assert(SMEM_ALLOC <= 232448, "exceeds the 227 KB per-block shared memory limit");
static_assert(P_L + 64 * LSTRIDE * 4 <= P_TPP, "L scratch overlaps T''");

// barrier slots
enum { B_Q = 0, B_K = 1, B_V = 2, B_Z = 3, B_MMA = 4, B_FULL = 5 /* chain: NP slots */, B_EMPTY = 5 /* prep */ };
constexpr int NBAR = B_FULL + NP;

// ---- TMEM
// chain: [0,128) C12 [hi | lo] -> v_new^T hi/lo [0,64) + (v_new e^{cL-c})^T hi/lo [64,128);
//        [128,192) S^T q^T; [192,256) v_new^T M^T; [256,384) dS^T; [384,512) S^T hi/lo (A operand)
constexpr uint32_t T_V = 0, T_VN_HI = 0, T_VN_LO = 32, T_VP_HI = 64, T_VP_LO = 96, T_O = 128, T_O2 = 192,
                   T_S = 256, T_SA_HI = 384, T_SA_LO = 448;
// prep: [0,64) P1; [128,256) P3 [T''_hi | T''_lo] parts of W^T
constexpr uint32_t T_P = 0, T_W = 128;

__global__ void __launch_bounds__(NTHREADS, 1) gdn_prefill_split_kernel(const __grid_constant__ Params p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    const uint32_t sb = ptx::smem_u32(smem);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int quarter = warp & 3, half = warp >> 2;
    const int row = quarter * 32 + lane;
    const uint32_t rank = ptx::cluster_ctarank();
    const bool chain = (rank == 0);
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
    const long long tok_base = (long long)bcoord * p.T + t_begin;

    const uint32_t misc_off = chain ? C_MISC : P_MISC;
    float* misc = reinterpret_cast<float*>(smem + misc_off);
    float* c_s = misc + M_C / 4;
    float* beta_s = misc + M_BETA / 4;
    float* w_s = misc + M_W / 4;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + misc_off + M_FLAG);
    const uint32_t bar0 = sb + misc_off + M_BAR;
    auto bar = [&](int i) { return bar0 + 8u * (uint32_t)i; };
    const uint32_t tmem_cols = chain ? 512u : 256u;

    if (tid == 0) {
        for (int i = 0; i < NBAR; ++i) ptx::mbar_init(bar(i), 1);
        ptx::fence_mbar_init();
        *abort_flag = 0;
    }
    if (warp == 0) {
        ptx::tmem_alloc(sb + misc_off + M_TMEM, tmem_cols);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + misc_off + M_TMEM);
    const uint32_t tl = tmem + ((uint32_t)(quarter * 32) << 16);

    uint32_t issued[NBAR] = {}, consumed[NBAR] = {};
    auto fail = [&]() {
        *abort_flag = 1;
        if (p.status) atomicOr(p.status, 1u);
    };
    auto wait_bar = [&](int i, uint32_t parity) {
        if (ptx::mbar_wait(bar(i), parity, WAIT_ITERS)) ++consumed[i];
        else fail();
    };
    auto wait_mma = [&]() {
        wait_bar(B_MMA, consumed[B_MMA] & 1u);
        ptx::tc_fence_after();
    };
    auto commit = [&]() {
        ptx::mma_commit(bar(B_MMA));
        ++issued[B_MMA];
    };
    auto load_tile = [&](int b, uint32_t dst, const CUtensorMap* map, int head, int n) {
        ++issued[b];
        ptx::mbar_arrive_expect_tx(bar(b), 16384);
        const int t = t_begin + n * CS;
        ptx::tma_load_4d(sb + dst, map, bar(b), 0, head, t, bcoord);
        ptx::tma_load_4d(sb + dst + (dst == C_QK || dst == C_QK + 8192 ? 16384 : 8192), map, bar(b), 64, head, t,
                         bcoord);
    };
    // q -> rows 0-63 and k -> rows 64-127 of the 128-row qk panels; v, z -> 64-row panels
    auto load_q = [&](int n) { load_tile(B_Q, C_QK, &p.tm_q, hq, n); };
    auto load_k = [&](int n) { load_tile(B_K, C_QK + 8192, &p.tm_k, hq, n); };

    constexpr uint32_t ID_P = ptx::idesc_bf16(128, 64, 0, 0, 0);
    constexpr uint32_t ID_W = ptx::idesc_bf16(128, 128, 1, 0, 0);
    constexpr uint32_t ID_U = ptx::idesc_bf16(128, 128, 1, 0, 0);
    constexpr uint32_t ID_WS = ptx::idesc_bf16(128, 128, 0, 1, 1);
    constexpr uint32_t ID_O = ptx::idesc_bf16(128, 64, 0, 0, 0);
    constexpr uint32_t ID_S = ptx::idesc_bf16(128, 128, 0, 1, 0);

    if (chain) {
        // ============================== chain CTA ==============================
        float S[64];
        auto store_state_operand = [&]() {
#pragma unroll
            for (int c2 = 0; c2 < 2; ++c2) {
                uint32_t hi[16], lo[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) split2(S[32 * c2 + 2 * j], S[32 * c2 + 2 * j + 1], hi[j], lo[j]);
                ptx::tmem_st16(tl + T_SA_HI + 32 * half + 16 * c2, hi);
                ptx::tmem_st16(tl + T_SA_LO + 32 * half + 16 * c2, lo);
            }
        };
        {
            const size_t sbase = ((size_t)seq * p.HV + h) * HD * HD;
#pragma unroll
            for (int j = 0; j < 64; ++j) {
                const int dk = 64 * half + j;
                S[j] = (p.s0 != nullptr) ? p.s0[sbase + (size_t)dk * HD + row] : 0.f;
            }
            store_state_operand();
        }
        if (tid < HD) w_s[tid] = p.gated ? __bfloat162float(p.w[tid]) : 0.f;
        const int et = tid >> 2, eq = tid & 3;
        auto load_v = [&](int n) { load_tile(B_V, C_V, &p.tm_v, h, n); };
        auto load_z = [&](int n) { load_tile(B_Z, C_Z, &p.tm_z, h, n); };
        if (tid == 0) {
            for (int s = 0; s < NP; ++s) {  // arm the slots for the first chunk of each prep CTA
                ++issued[B_FULL + s];
                ptx::mbar_arrive_expect_tx(bar(B_FULL + s), SL_BYTES);
            }
        }
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        ptx::cluster_sync();  // every CTA's barriers are initialised and the slots armed
        ptx::tc_fence_after();
        if (tid == 0 && NC > 0) {
            load_q(0);
            load_k(0);
            load_v(0);
            if (p.gated) load_z(0);
        }

        for (int n = 0; n < NC; ++n) {
            if (*abort_flag) break;
            const int valid = min(CS, len - n * CS);
            const long long tok0 = tok_base + (long long)n * CS;
            const uint32_t ph = (uint32_t)(n & 1);
            const int slot = n % NP;
            const uint32_t sp = C_SLOT + slot * SLOT;
            const float* ec_s = reinterpret_cast<const float*>(smem + sp + SL_EC);
            const float* ed_s = reinterpret_cast<const float*>(smem + sp + SL_ED);

            // ---- C12: v_new^T = v^T [T'_hi;T'_lo]^T - S^T [W_hi|W_lo] (hi terms cols 0-63, lo 64-127)
            if (!ptx::mbar_wait_cluster(bar(B_FULL + slot), (uint32_t)((n / NP) & 1), WAIT_ITERS)) fail();
            else ++consumed[B_FULL + slot];
            wait_bar(B_V, ph);
            if (tid == 0) {
                ptx::tc_fence_after();
#pragma unroll
                for (int s = 0; s < 4; ++s) {
                    const uint64_t a = ptx::sw128_desc(sb + C_V + s * 2048, 8192, 1024);
                    const uint64_t b = ptx::sw128_desc(sb + sp + SL_TP + s * 32, 16, 1024);
                    ptx::mma_bf16(tmem + T_V, a, b, ID_U, s > 0);
                }
#pragma unroll
                for (int part = 0; part < 2; ++part) {
                    const uint32_t sa = part ? T_SA_LO : T_SA_HI;
#pragma unroll
                    for (int s = 0; s < 8; ++s) {
                        const uint64_t b = ptx::sw128_desc(sb + sp + SL_W + s * 2048, 16384, 1024);
                        ptx::mma_bf16_ts(tmem + T_V, tmem + sa + 8 * s, b, ID_WS, 1u);
                    }
                }
                commit();
            }
            wait_mma();
            if (tid == 0 && n + 1 < NC) load_v(n + 1);
            {   // v_new hi/lo and (v_new e^{cL-c}) hi/lo -> TMEM A operands
                float v[32];
                {
                    float v2[32];
                    ptx::tmem_ld32(tl + T_V + 32 * half, v);
                    ptx::tmem_ld32(tl + T_V + 64 + 32 * half, v2);
                    ptx::tmem_wait_ld();
#pragma unroll
                    for (int jj = 0; jj < 32; ++jj) v[jj] += v2[jj];
                }
                uint32_t vh[16], vl[16], ph_[16], pl[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    split2(v[2 * j], v[2 * j + 1], vh[j], vl[j]);
                    split2(v[2 * j] * ed_s[32 * half + 2 * j], v[2 * j + 1] * ed_s[32 * half + 2 * j + 1], ph_[j], pl[j]);
                }
                ptx::tc_fence_before();
                __syncthreads();  // all of cols [0,128) read before they are overwritten
                ptx::tc_fence_after();
                ptx::tmem_st16(tl + T_VN_HI + 16 * half, vh);
                ptx::tmem_st16(tl + T_VN_LO + 16 * half, vl);
                ptx::tmem_st16(tl + T_VP_HI + 16 * half, ph_);
                ptx::tmem_st16(tl + T_VP_LO + 16 * half, pl);
                ptx::tmem_wait_st();
            }
            ptx::tc_fence_before();
            __syncthreads();
            if (*abort_flag) break;

            // ---- C3 / C4
            wait_bar(B_Q, ph);
            wait_bar(B_K, ph);
            if (tid == 0) {
                ptx::tc_fence_after();
#pragma unroll
                for (int part = 0; part < 2; ++part) {
                    const uint32_t sa = part ? T_SA_LO : T_SA_HI;
#pragma unroll
                    for (int s = 0; s < 8; ++s) {
                        const uint64_t b =
                            ptx::sw128_desc(sb + C_QK + (s >> 2) * 16384 + (s & 3) * 32, 16, 1024);
                        ptx::mma_bf16_ts(tmem + T_O, tmem + sa + 8 * s, b, ID_O, (part | s) > 0);
                    }
                }
#pragma unroll
                for (int term = 0; term < 3; ++term) {
                    const uint32_t va = (term == 1) ? T_VN_LO : T_VN_HI;
                    const uint32_t mb = sp + SL_M + ((term == 2) ? 8192u : 0u);
#pragma unroll
                    for (int s = 0; s < 4; ++s) {
                        const uint64_t b = ptx::sw128_desc(sb + mb + s * 32, 16, 1024);
                        ptx::mma_bf16_ts(tmem + T_O2, tmem + va + 8 * s, b, ID_O, (term | s) > 0);
                    }
                }
#pragma unroll
                for (int part = 0; part < 2; ++part) {
                    const uint32_t va = part ? T_VP_LO : T_VP_HI;
#pragma unroll
                    for (int s = 0; s < 4; ++s) {
                        const uint64_t b = ptx::sw128_desc(sb + C_QK + 8192 + s * 2048, 16384, 1024);
                        ptx::mma_bf16_ts(tmem + T_S, tmem + va + 8 * s, b, ID_S, (part | s) > 0);
                    }
                }
                commit();
            }
            wait_mma();
            if (tid == 0 && n + 1 < NC) {
                load_q(n + 1);
                load_k(n + 1);
            }
            {   // S <- e^{cL} S + dS
                const float gam = ec_s[CS - 1];
#pragma unroll
                for (int c2 = 0; c2 < 2; ++c2) {
                    float v[32];
                    ptx::tmem_ld32(tl + T_S + 64 * half + 32 * c2, v);
                    ptx::tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 32; ++j) S[32 * c2 + j] = fmaf(gam, S[32 * c2 + j], v[j]);
                }
            }
            {   // o = scale e^c o1 + o2 -> bf16 staging
                float v[32], v2[32];
                ptx::tmem_ld32(tl + T_O + 32 * half, v);
                ptx::tmem_ld32(tl + T_O2 + 32 * half, v2);
                ptx::tmem_wait_ld();
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) v[jj] = fmaf(p.scale * ec_s[32 * half + jj], v[jj], v2[jj]);
                __nv_bfloat16* ot = reinterpret_cast<__nv_bfloat16*>(smem + C_OST);
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) ot[sw_off(32 * half + jj, row, 64) >> 1] = __float2bfloat16_rn(v[jj]);
            }
            store_state_operand();
            ptx::tmem_wait_st();
            ptx::tc_fence_before();
            __syncthreads();  // slot fully consumed, o staged, new S operand in TMEM
            if (tid == 0) {   // hand the slot back to its prep CTA
                if (n + NP < NC) {
                    ++issued[B_FULL + slot];
                    ptx::mbar_arrive_expect_tx(bar(B_FULL + slot), SL_BYTES);
                }
                // the prep CTA's barriers sit at its own misc offset
                ptx::mbar_arrive_remote(ptx::mapa(sb + P_MISC + M_BAR + 8u * B_EMPTY, (uint32_t)(1 + slot)));
            }

            // ---- epilogue: 4 threads per token, 16-byte chunks {eq, eq+4, eq+8, eq+12}
            {
                float o[32];
#pragma unroll
                for (int m = 0; m < 4; ++m) {
                    uint32_t w4[4];
                    ld_shared_v4(sb + C_OST + sw_chunk(et, eq + 4 * m, 64), w4[0], w4[1], w4[2], w4[3]);
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const __nv_bfloat162 b2 = *reinterpret_cast<const __nv_bfloat162*>(&w4[u]);
                        o[8 * m + 2 * u] = __bfloat162float(b2.x);
                        o[8 * m + 2 * u + 1] = __bfloat162float(b2.y);
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
                    wait_bar(B_Z, ph);
#pragma unroll
                    for (int m = 0; m < 4; ++m) {
                        const int c = eq + 4 * m;
                        uint32_t w4[4];
                        ld_shared_v4(sb + C_Z + sw_chunk(et, c, 64), w4[0], w4[1], w4[2], w4[3]);
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const int j = 8 * m + 2 * u, dv = 8 * c + 2 * u;
                            const __nv_bfloat162 z2 = *reinterpret_cast<const __nv_bfloat162*>(&w4[u]);
                            const float z0 = __low2float(z2), z1 = __high2float(z2);
                            const float y0 = (w_s[dv] * bf16r(o[j] * rstd)) * (z0 * rcpf(1.f + ex2f(-z0 * LOG2E)));
                            const float y1 =
                                (w_s[dv + 1] * bf16r(o[j + 1] * rstd)) * (z1 * rcpf(1.f + ex2f(-z1 * LOG2E)));
                            outw[4 * m + u] = pack_bf16(y0, y1);
                        }
                    }
                }
                if (et < valid) {
                    uint4* dst = reinterpret_cast<uint4*>(p.out + (size_t)(tok0 + et) * p.HV * HD + (size_t)h * HD);
#pragma unroll
                    for (int m = 0; m < 4; ++m)
                        dst[eq + 4 * m] = make_uint4(outw[4 * m], outw[4 * m + 1], outw[4 * m + 2], outw[4 * m + 3]);
                }
            }
            __syncthreads();
            if (tid == 0 && p.gated && n + 1 < NC) {
                ptx::fence_proxy_async_smem();
                load_z(n + 1);
            }
        }
        if (!*abort_flag) {
            const size_t sbase = ((size_t)seq * p.HV + h) * HD * HD;
#pragma unroll
            for (int j = 0; j < 64; ++j) p.sf[sbase + (size_t)(64 * half + j) * HD + row] = S[j];
        }
    } else {
        // ============================== prep CTA ==============================
        const int pi = (int)rank - 1;  // owns chunks pi, pi + NP, ...
        float* Ls = reinterpret_cast<float*>(smem + P_L);
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
        ptx::cluster_sync();
        if (tid == 0 && pi < NC) {
            load_q(pi);
            load_k(pi);
        }
        if (warp == 0 && pi < NC) load_gates(pi);

        int k = 0;
        for (int n = pi; n < NC; n += NP, ++k) {
            if (*abort_flag) break;
            const uint32_t stg = P_STG + (uint32_t)(k & 1) * SLOT;
            float* ec_s = reinterpret_cast<float*>(smem + stg + SL_EC);
            float* ed_s = reinterpret_cast<float*>(smem + stg + SL_ED);
            float* X = reinterpret_cast<float*>(smem + stg + SL_W);  // inversion scratch (W area not yet written)
            const uint32_t ph = (uint32_t)(k & 1);
            __syncthreads();  // thread 0 has confirmed that staging[k & 1] was shipped and consumed

            if (warp == 0) {
                const float g0 = gn0, g1 = gn1, b0 = bn0, b1 = bn1;
                if (n + NP < NC) load_gates(n + NP);
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
            wait_bar(B_Q, ph);
            wait_bar(B_K, ph);
            if (tid == 0) {
                ptx::tc_fence_after();
#pragma unroll
                for (int s = 0; s < 8; ++s) {
                    const uint32_t koff = (uint32_t)(s >> 2) * 16384u + (uint32_t)(s & 3) * 32u;
                    const uint64_t a = ptx::sw128_desc(sb + P_QK + koff, 16, 1024);
                    const uint64_t b = ptx::sw128_desc(sb + P_QK + 8192 + koff, 16, 1024);
                    ptx::mma_bf16(tmem + T_P, a, b, ID_P, s > 0);
                }
                commit();
            }
            __syncthreads();
            wait_mma();
            {   // rows 0-63: M (hi/lo -> staging); rows 64-127: L
                float v[32];
                ptx::tmem_ld32(tl + T_P + 32 * half, v);
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
                        put8_split(sb + stg + SL_M + co, sb + stg + SL_M + 8192 + co, m + 8 * ch, true);
                    }
                } else {
                    const int i = row - CS;
                    const float ci = c_s[i], bi = beta_s[i];
                    float* lrow = Ls + i * LSTRIDE + 32 * half;
#pragma unroll
                    for (int j4 = 0; j4 < 8; ++j4) {
                        float4 o4;
                        float* o = reinterpret_cast<float*>(&o4);
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const int jj = 4 * j4 + u, j = 32 * half + jj;
                            o[u] = (j < i) ? bi * v[jj] * ex2f((ci - c_s[j]) * LOG2E) : 0.f;
                        }
                        *reinterpret_cast<float4*>(lrow + 4 * j4) = o4;
                    }
                }
            }
            ptx::tc_fence_before();
            __syncthreads();
            invert_unit_lower(Ls, X, tid, [](int) {});
            {   // T' -> staging (stacked hi/lo), T'' -> local
                const int i = tid >> 2, jb = tid & 3;
                float tp[16], tpp[16];
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) {
                    const float4 t4 = ld4(Ls + i * LSTRIDE + 16 * jb + 4 * q4);
                    const float tt[4] = {t4.x, t4.y, t4.z, t4.w};
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int jj = 4 * q4 + u, j = 16 * jb + jj;
                        tp[jj] = tt[u] * beta_s[j];
                        tpp[jj] = tp[jj] * ec_s[j];
                    }
                }
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                    const uint32_t co = sw_chunk(i, 2 * jb + hh, 64);
                    put8_split(sb + stg + SL_TP + co, sb + stg + SL_TP + 8192 + co, tp + 8 * hh, true);
                    put8_split(sb + P_TPP + co, sb + P_TPP + 8192 + co, tpp + 8 * hh, true);
                }
            }
            ptx::fence_proxy_async_smem();
            __syncthreads();
            if (tid == 0) {  // P3: W^T = K^T [T''_hi; T''_lo]^T
                ptx::tc_fence_after();
#pragma unroll
                for (int s = 0; s < 4; ++s) {
                    const uint64_t a = ptx::sw128_desc(sb + P_QK + 8192 + s * 2048, 16384, 1024);
                    const uint64_t b = ptx::sw128_desc(sb + P_TPP + s * 32, 16, 1024);
                    ptx::mma_bf16(tmem + T_W, a, b, ID_W, s > 0);
                }
                commit();
            }
            wait_mma();
            if (tid == 0 && n + NP < NC) {  // q and k consumed: fetch this CTA's next chunk
                load_q(n + NP);
                load_k(n + NP);
            }
            {   // W^T rows (dk = row) -> staging, hi and lo tiles 16 KB apart
                float v[32], v2[32];
                ptx::tmem_ld32(tl + T_W + 32 * half, v);
                ptx::tmem_ld32(tl + T_W + 64 + 32 * half, v2);
                ptx::tmem_wait_ld();
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) v[jj] += v2[jj];
#pragma unroll
                for (int ch = 0; ch < 4; ++ch) {
                    const uint32_t co = sw_chunk(row, 4 * half + ch, 128);
                    put8_split(sb + stg + SL_W + co, sb + stg + SL_W + 16384 + co, v + 8 * ch, true);
                }
            }
            ptx::tc_fence_before();
            ptx::fence_proxy_async_smem();
            __syncthreads();
            if (tid == 0) {  // ship to the chain CTA once it has consumed this CTA's previous chunk
                if (k >= 1) {
                    if (ptx::mbar_wait_cluster(bar(B_EMPTY), (uint32_t)((k - 1) & 1), WAIT_ITERS)) ++consumed[B_EMPTY];
                    else fail();
                }
                const uint32_t dst = ptx::mapa(sb + C_SLOT + (uint32_t)pi * SLOT, 0);
                const uint32_t fb = ptx::mapa(sb + C_MISC + M_BAR + 8u * (uint32_t)(B_FULL + pi), 0);
                ptx::bulk_copy_s2cluster(dst, sb + stg, 65536, fb);
                ptx::bulk_copy_s2cluster(dst + 65536, sb + stg + 65536, SL_BYTES - 65536, fb);
            }
        }
        if (tid == 0 && k >= 1 && !*abort_flag) {  // the last shipment must land before this CTA exits
            if (ptx::mbar_wait_cluster(bar(B_EMPTY), (uint32_t)((k - 1) & 1), WAIT_ITERS)) ++consumed[B_EMPTY];
            else fail();
        }
    }

    if (*abort_flag && tid == 0) {
#pragma unroll
        for (int i = 0; i < 5; ++i)
            while (consumed[i] < issued[i]) {
                ptx::mbar_wait(bar(i), consumed[i] & 1u, WAIT_ITERS);
                ++consumed[i];
            }
    }
    ptx::tc_fence_before();
    ptx::cluster_sync();  // no CTA leaves while a peer may still touch its shared memory
    if (warp == 0) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem, tmem_cols);
    }
}

}  // namespace split

cudaError_t launch_split(const Params& p, int nseq, int HV, cudaStream_t stream) {
    static bool attr_done[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 64 && !attr_done[dev]) {
        e = cudaFuncSetAttribute(split::gdn_prefill_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)split::SMEM_ALLOC);
        if (e != cudaSuccess) return e;
        attr_done[dev] = true;
    }
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(1 + split::NP, HV, nseq);
    cfg.blockDim = dim3(split::NTHREADS, 1, 1);
    cfg.dynamicSmemBytes = split::SMEM_ALLOC;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1 + split::NP;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, split::gdn_prefill_split_kernel, p);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

int split_cluster_ctas() { return 1 + split::NP; }

}  // namespace gdn
