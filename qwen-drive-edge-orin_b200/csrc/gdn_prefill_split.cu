// Cluster-split variant of the chunked gated-delta-rule prefill for small
// batches (few (sequence, v-head) units relative to the 148 SMs).
//
// Each (sequence, v-head) runs on a cluster of NP + 2 CTAs:
//   * rank 0, the chain CTA, owns the recurrent state and runs only the
//     state-dependent steps of every chunk: C12 (v_new), C3/C4 (output and
//     state increment) and the state update, and stages o as bf16;
//   * ranks 2..NP+1, the prep CTAs, run the state-independent chunk math for
//     chunks n = rank-2, rank-2+NP, ...: gates, P1 ([Q;K]K^T), L and M, the
//     triangular inverse, T' and T'', P3 (W), and ship them into the chain
//     CTA's slot buffers with shared-to-shared bulk copies (completing on the
//     chain's mbarriers; no multicast). A slot has two parts that are handed
//     back separately: part A (T', W, decay factors) once C12 has read it,
//     part B (M) once the intra-chunk output term has;
//   * rank 1, the output CTA, receives each chunk's staged o the same way
//     and runs the gated-RMSNorm epilogue (z tiles, norm weight, y stores).
// Prep, chain and output work of different chunks overlap, so the chain's
// period per chunk is its own work only.
//
// Inside the chain CTA the work is split by warp. A tcgen05.mma issue does
// not return before the tensor core has (nearly) executed the instruction,
// so the issuing warp is busy for the whole MMA time; warp 8 does only that,
// warp 9 issues the TMA loads and hands slot parts back as soon as their
// buffers are free, and warps 0-7 read and write TMEM and run the CUDA-core
// steps. Per chunk n the issue order is C12(n) (its state-independent half
// first), S^T q^T(n), then - once warps 0-7 have formed the v_new operands -
// dS(n) and v_new^T M^T(n); warps 0-7 form v_new(n), update the state, then
// read the output back and stage it, which overlaps C12 and S^T q^T of chunk
// n+1. The hand-offs between the groups are mbarriers with bounded waits.
//
// The math, precision scheme and operand layouts are those of
// gdn_prefill_kernel (gdn_prefill.cu).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <atomic>

#include "gdn_common.cuh"
#include "gdn_prefill.h"
#include "sm100_ptx.cuh"

namespace gdn {
namespace split {

constexpr int NCOMPUTE = 256;             // warpgroups 0-1: TMEM and CUDA-core work
constexpr int NTHREADS = NCOMPUTE + 128;  // warpgroup 2 (chain CTA): warp 8 MMA issue, warp 9 TMA / slots
constexpr int ISSUER_WARP = NCOMPUTE / 32;
// Registers: 168 per thread at launch (384 threads fill the 64K file); warpgroup 2 gives
// part of its share to warpgroups 0-1: 2 x 128 x 192 + 128 x 120 = 384 x 168. The MMA
// warp keeps the unrolled MMA descriptors in registers, hence its 120.
constexpr int LAUNCH_REGS = 168, COMPUTE_REGS = 192, ISSUE_REGS = 120;
static_assert(2 * 128 * COMPUTE_REGS + 128 * ISSUE_REGS <= NTHREADS * LAUNCH_REGS, "register split exceeds the pool");
constexpr uint32_t CSYNC = 1;            // named barrier of warps 0-7
constexpr uint32_t GSYNC = 2;            // named barrier of warpgroup 2 (output CTA: the gate warps)
constexpr int NP = 2;                    // prep CTAs per cluster
// Cluster ranks 2r and 2r+1 land on neighbouring SMs (one TPC). The kernel is sensitive to
// instruction fetch (its hot loops exceed an SM's instruction cache), and it ran faster
// with the two prep CTAs (the same code) on one pair and the chain and output CTAs on the
// other than with the chain and a prep CTA paired (config 1: 83.3 -> 80.0 us).
// Every cross-CTA address (mapa target, slot, barrier) names its CTA by one of these constants;
// a CTA's own layout (C_*, P_*, U_* offsets and its barriers) is fixed by its role, so a peer's
// barrier or slot is only valid at the rank that runs that role.
constexpr uint32_t CHAIN_RANK = 0;       // the chain CTA
constexpr uint32_t OUT_RANK = 1;         // the output CTA
constexpr uint32_t PREP_RANK0 = 2;       // prep CTAs: ranks 2 .. NP + 1
constexpr int CLUSTER = NP + 2;          // chain, NP prep CTAs, output
static_assert(CHAIN_RANK != OUT_RANK && (CHAIN_RANK < PREP_RANK0 || CHAIN_RANK >= PREP_RANK0 + NP) &&
                  (OUT_RANK < PREP_RANK0 || OUT_RANK >= PREP_RANK0 + NP) && CHAIN_RANK < CLUSTER &&
                  OUT_RANK < CLUSTER && PREP_RANK0 + NP <= CLUSTER,
              "the roles must take distinct ranks of the cluster");

// ---- prep CTA staging layout (one chunk's shipment)
constexpr uint32_t SL_TP = 0;        // [T'_hi; T'_lo] 128 rows x 64 cols bf16 (K-major, stacked along N)
constexpr uint32_t SL_W = 16384;     // W^T hi, lo: [128 dk][64 tok] bf16 MN-major tiles, 16 KB apart
constexpr uint32_t SL_M = 49152;     // M hi, lo: [64][64] bf16, 8 KB apart
constexpr uint32_t SL_EC = 65536;    // e^c      [64] f32
constexpr uint32_t SL_ED = 65792;    // e^{cL-c} [64] f32
constexpr uint32_t SLOT = 66560;     // staging stride (1024-aligned)
static_assert(SL_ED == SL_EC + 4 * CS, "e^{cL-c} follows e^c (one copy moves both)");
// ---- chain CTA slot layout: part A = staging [SL_TP, SL_M) + [SL_EC, SL_EC + 512), part B = M
constexpr uint32_t A_TP = 0, A_W = 16384, A_EC = 49152, A_ED = 49408;
constexpr uint32_t A_BYTES = 49664;
constexpr uint32_t ASLOT = 50176;    // 1024-aligned stride
constexpr uint32_t B_BYTES = 16384;
constexpr int NSLOT = 2;             // slot s is filled by prep CTA 1 + s
static_assert(NSLOT == NP, "each prep CTA owns one chain slot");

constexpr uint32_t O_BYTES = 16384;  // o of one chunk: [64 tok][128 dv] bf16, two 64-row panels of 8 KB

// ---- chain CTA shared memory
constexpr uint32_t C_QK = 0;          // q rows 0-63 | k rows 64-127 (16 KB/panel)
constexpr uint32_t C_V = 32768;
constexpr uint32_t C_OST = 49152;     // 2 o staging buffers (chunk parity), shipped to the output CTA
constexpr uint32_t C_ASLOT = C_OST + 2 * O_BYTES;       // NSLOT part-A slots
constexpr uint32_t C_BSLOT = C_ASLOT + NSLOT * ASLOT;   // NSLOT part-B slots (M)
constexpr uint32_t C_MISC = C_BSLOT + NSLOT * B_BYTES;
// ---- prep CTA shared memory
constexpr uint32_t P_QK = 0;
constexpr uint32_t P_L = 32768;                  // L / T fp32 [64][68]
constexpr uint32_t P_TPP = 50176;                // T'' hi, lo [64][64] bf16
constexpr uint32_t P_STG = 66560;                // 2 staging slots
constexpr uint32_t P_GATE = P_STG + 2 * SLOT;    // 2 gate slots (chunk parity): c, beta, e^c, e^{cL-c} [64] f32
constexpr uint32_t GSLOT = 1024;
constexpr uint32_t P_MISC = P_GATE + 2 * GSLOT;
// ---- output CTA shared memory
constexpr uint32_t U_OSLOT = 0;                  // 2 o^T slots (chunk parity), filled by the chain CTA
constexpr uint32_t U_Z = 2 * O_BYTES;            // 2 z tiles (chunk parity)
constexpr uint32_t U_OT = U_Z + 2 * O_BYTES;     // o [64 tok][128 dv] (two 64-row panels), transposed here
constexpr uint32_t U_GATE = U_OT + O_BYTES;      // 2 gate tiles (chunk parity): w * silu(z) fp32 [64 tok][128 dv],
constexpr uint32_t GATE_BYTES = 2 * O_BYTES;     //   16-byte chunks swizzled
constexpr uint32_t U_MISC = U_GATE + 2 * GATE_BYTES;
// ---- misc (all roles; the chain keeps e^c of chunks with even / odd index at M_C, 128 floats)
constexpr uint32_t M_C = 0, M_W = 512, M_BAR = 1024, M_TMEM = 1280, M_FLAG = 1284, M_DONE = 1288,
                   M_BYTES = 1408;
constexpr uint32_t MAX2(uint32_t a, uint32_t b) { return a > b ? a : b; }
constexpr uint32_t SMEM_BYTES = MAX2(MAX2(C_MISC, P_MISC), U_MISC) + M_BYTES;
constexpr uint32_t SMEM_ALLOC = SMEM_BYTES + 1024;
static_assert(SMEM_ALLOC <= 232448, "exceeds the 227 KB per-block shared memory limit");
static_assert(P_L + 64 * LSTRIDE * 4 <= P_TPP, "L scratch overlaps T''");

// barrier slots: TMA tiles; MMA commit groups (chain: B_VT = v^T T'^T, the part of C12 that
// reads the v tile, B_MMA = C12, X1 = S^T q^T + dS, Y = v_new^T M^T; B_DRAIN only on the
// abort path); chain hand-offs from warps 0-7 to the
// MMA / producer warps (one arrival per thread): v_new operands formed, new state operand stored,
// output accumulators read. Per role, the barriers from B_FULLA up: chain - slot parts filled
// by the prep CTAs, o staging buffers handed back by the output CTA; prep - slot parts handed
// back; output - o slots filled by the chain CTA, z tiles loaded.
enum {
    B_Q = 0, B_K = 1, B_V = 2, B_MMA = 3, B_X1 = 4, B_Y = 5, B_DRAIN = 6,
    B_VNR = 7, B_SOP = 8, B_OFREE = 9, B_VT = 10,
    B_FULLA = 11 /* chain: NSLOT */, B_FULLB = B_FULLA + NSLOT /* chain: NSLOT */,
    B_EMPTYO = B_FULLB + NSLOT /* chain: 2 */,
    B_X2 = B_EMPTYO + 2 /* chain: S^T q^T done */, B_DRAIN2 = B_X2 + 1 /* chain: output-MMA warp, abort path */,
    B_TSFREE = B_DRAIN2 + 1 /* chain: dS read by the state update (one arrival per thread) */,
    B_EMPTYA = 11 /* prep */, B_EMPTYB = 12 /* prep */,
    B_GREADY = 13 /* prep: 2, gate slot written (32 arrivals) */, B_GFREE = 15 /* prep: 2, gate slot read */,
    B_FULLO = 11 /* output: 2 */, B_ZT = 13 /* output: 2 */,
    B_OGFULL = 15 /* output: 2, gate tile written */, B_OGFREE = 17 /* output: 2, gate tile read */
};
constexpr int NBAR = B_TSFREE + 1;
static_assert(B_GFREE + 2 <= NBAR && B_OGFREE + 2 <= NBAR, "prep and output barriers exceed the barrier area");
static_assert(M_BAR + 8 * NBAR <= M_TMEM, "barriers overlap the TMEM address word");

// ---- TMEM
// chain: [0,128) v_new^T hi/lo [0,64) + (v_new e^{cL-c})^T hi/lo [64,128) (A operands);
//        [128,192) S^T q^T; [192,256) v_new^T M^T; [256,384) C12 [hi | lo], then dS^T; [384,512)
//        S^T hi/lo (A operand). C12 of chunk n+1 may start once the state update has read dS of
//        chunk n, and the v_new operands are not written over their own input.
constexpr uint32_t T_VN_HI = 0, T_VN_LO = 32, T_VP_HI = 64, T_VP_LO = 96, T_O = 128, T_O2 = 192,
                   T_S = 256, T_C12 = T_S, T_SA_HI = 384, T_SA_LO = 448;
// prep: [0,64) P1; [128,256) P3 [T''_hi | T''_lo] parts of W^T
constexpr uint32_t T_P = 0, T_W = 128;

// A bounded wait that ran out: set the CTA's abort flag and record bit 0 plus the role that gave up
// in the status word. Out of line: it runs only after a timeout, and inlined at each of the kernel's
// many wait sites it would put cold code between the hot loops' instructions (the kernel is
// sensitive to instruction fetch).
__device__ __noinline__ void record_failure(volatile int* abort_flag, unsigned int* status) {
    *abort_flag = 1;
    if (status) {  // the role, from the thread and the CTA's rank
        const uint32_t w = threadIdx.x >> 5, r = ptx::cluster_ctarank();
        const uint32_t role = r == CHAIN_RANK ? (w < (uint32_t)ISSUER_WARP ? 8u : 9u + (w - ISSUER_WARP))
                                              : (r == OUT_RANK ? 14u : (w < (uint32_t)ISSUER_WARP ? 12u : 13u));
        atomicOr(status, 1u | (1u << role));
    }
}

// kSeg: the instantiation for the passes of a segmented call (segment indexing, the state
// pass's identity runs, last-segment final states); the plain instantiation carries none of it.
template <bool kSeg>
__global__ void __launch_bounds__(NTHREADS, 1) gdn_prefill_split_kernel(const __grid_constant__ Params p) {
    // the tensor maps are kernel parameters, not data of the previous launch: fetch them while it ends
    if (threadIdx.x == 0) {
        ptx::prefetch_tensormap(&p.tm_q);
        ptx::prefetch_tensormap(&p.tm_k);
        ptx::prefetch_tensormap(&p.tm_v);
        if (p.gated) ptx::prefetch_tensormap(&p.tm_z);
        if (kSeg && (int)blockIdx.y >= p.HV) ptx::prefetch_tensormap(&p.tm_v0);
    }
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    const uint32_t sb = ptx::smem_u32(smem);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool compute = (warp < ISSUER_WARP);
    const int quarter = warp & 3, half = (warp >> 2) & 1;  // TMEM lane quarter / column half (warps 0-7)
    const int row = quarter * 32 + lane;
    const uint32_t rank = ptx::cluster_ctarank();
    const bool chain = (rank == CHAIN_RANK);
    const bool outcta = (rank == OUT_RANK);
    // state pass of a segmented call: y >= HV runs head y - HV from the identity with zero v
    const bool phi_unit = kSeg && (int)blockIdx.y >= p.HV;
    const int h = phi_unit ? (int)blockIdx.y - p.HV : (int)blockIdx.y;
    const int seq = blockIdx.z;
    const int hq = h / (p.HV / p.HQK);

    const uint32_t misc_off = chain ? C_MISC : (outcta ? U_MISC : P_MISC);
    float* misc = reinterpret_cast<float*>(smem + misc_off);
    float* w_s = misc + M_W / 4;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + misc_off + M_FLAG);
    volatile int* done_flag = reinterpret_cast<volatile int*>(smem + misc_off + M_DONE);
    const uint32_t bar0 = sb + misc_off + M_BAR;
    auto bar = [&](int i) { return bar0 + 8u * (uint32_t)i; };
    const uint32_t tmem_cols = chain ? 512u : (outcta ? 0u : 256u);

    if (tid == 0) {
        for (int i = 0; i < NBAR; ++i)
            ptx::mbar_init(bar(i), (chain && ((i >= B_VNR && i <= B_OFREE) || i == B_TSFREE)) ? (uint32_t)NCOMPUTE
                                   : (!chain && !outcta && (i == B_GREADY || i == B_GREADY + 1)) ? 32u
                                                                                               : 1u);
        ptx::fence_mbar_init();
        *abort_flag = 0;
        *done_flag = 0;
    }
    if (warp == 0 && tmem_cols > 0) {
        ptx::tmem_alloc(sb + misc_off + M_TMEM, tmem_cols);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    // barriers, TMEM and the tensor maps above touch no global data; inputs may come from the
    // previous launch in the stream, so everything below waits for it
    ptx::grid_dependency_wait();
    ptx::grid_launch_dependents();
    int t_begin, len, bcoord;
    if (kSeg) {  // segment seq % seg_per_seq of batch row seq / seg_per_seq
        bcoord = seq / p.seg_per_seq;
        t_begin = (seq - bcoord * p.seg_per_seq) * p.seg_chunks * CS;
        len = min(p.seg_chunks * CS, p.T - t_begin);
    } else if (p.cu_seqlens != nullptr) {
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
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + misc_off + M_TMEM);
    const uint32_t tl = tmem + ((uint32_t)(quarter * 32) << 16);

    // Every wait names its phase parity, derived from the chunk index. The only counts kept
    // are of the TMA tiles and slot fills a thread arms (scalars, for the abort-path drain):
    // counters in an array indexed by slot parity would live in local memory, and with most
    // of the SM's L1 given to shared memory each update is a round trip to L2.
    //
    // Abort protocol. A wait that runs out sets the CTA's flag and records its role in the
    // status word (bit 0, plus 8-11: chain compute / MMA / load / output-MMA warps, 12-13: prep
    // compute / gate warps, 14: output CTA). Once the flag is set, no thread of the CTA arms a
    // barrier or issues a TMA load, MMA or bulk copy that it has not issued already: the phase
    // a failed wait was for may still be pending, and arming a pending phase (an arrival it has
    // no count for) or shipping into a peer's slot that was not armed is undefined. Single-
    // thread roles leave their loop at once; warps 0-7, which share named barriers, carry on to
    // their next vote (their own arrivals are on count barriers without transaction bytes) and
    // leave together.
    auto fail = [&]() { record_failure(abort_flag, p.status); };
    auto wait_bar = [&](int i, uint32_t parity) -> bool {
        if (ptx::mbar_wait_compact(bar(i), parity, WAIT_ITERS)) return true;
        fail();
        return false;
    };
    auto wait_mma = [&](uint32_t parity) -> bool {
        const bool ok = wait_bar(B_MMA, parity);
        ptx::tc_fence_after();
        return ok;
    };
    auto commit_to = [&](int b) { ptx::mma_commit(bar(b)); };
    // abort path: wait (bounded) for the last phase armed on a barrier (re-armed only after
    // its previous phase was consumed), and for every MMA this thread issued
    auto drain = [&](int b, uint32_t armed) {
        if (armed > 0) ptx::mbar_wait_compact(bar(b), (armed - 1) & 1u, WAIT_ITERS);
    };
    auto drain_mma = [&](int b) {
        ptx::mma_commit(bar(b));
        ptx::mbar_wait_compact(bar(b), 0u, WAIT_ITERS);
    };
    auto commit = [&]() { commit_to(B_MMA); };
    auto csync = [] { ptx::named_sync(CSYNC, NCOMPUTE); };
    // exit decision of warps 0-7: the OR of every thread's view of the flag, taken at a barrier
    auto vote_abort = [&] { return ptx::named_sync_or(CSYNC, NCOMPUTE, *abort_flag != 0); };
    // warps 0-7 -> warpgroup 2 hand-off, after this thread's TMEM accesses have completed
    auto hand_off = [&](int b) {
        ptx::tc_fence_before();
        ptx::mbar_arrive(bar(b));
    };
    auto load_tile = [&](int b, uint32_t dst, const CUtensorMap* map, int head, int n, uint32_t& armed) {
        ++armed;
        ptx::mbar_arrive_expect_tx(bar(b), 16384);
        const int t = t_begin + n * CS;
        ptx::tma_load_4d(sb + dst, map, bar(b), 0, head, t, bcoord);
        ptx::tma_load_4d(sb + dst + (dst == C_QK || dst == C_QK + 8192 ? 16384 : 8192), map, bar(b), 64, head, t,
                         bcoord);
    };
    // q -> rows 0-63 and k -> rows 64-127 of the 128-row qk panels; v, z -> 64-row panels
    // phases armed by this thread: q, k, v tiles; z tiles, slot parts A and B, o slots by parity
    uint32_t armed_q = 0, armed_k = 0, armed_v = 0, armed_z0 = 0, armed_z1 = 0;
    uint32_t armed_a0 = 0, armed_a1 = 0, armed_b0 = 0, armed_b1 = 0, armed_o0 = 0, armed_o1 = 0;
    auto load_q = [&](int n) { load_tile(B_Q, C_QK, &p.tm_q, hq, n, armed_q); };
    auto load_k = [&](int n) { load_tile(B_K, C_QK + 8192, &p.tm_k, hq, n, armed_k); };
    auto load_v = [&](int n) { load_tile(B_V, C_V, phi_unit ? &p.tm_v0 : &p.tm_v, h, n, armed_v); };
    // L2 prefetch of a later chunk's tile (both 64-column boxes), so that its TMA load is an L2 hit
    auto prefetch_tile = [&](const CUtensorMap* map, int head, int n) {
        if (n * CS >= len) return;
        const int t = t_begin + n * CS;
        ptx::tma_prefetch_4d(map, 0, head, t, bcoord);
        ptx::tma_prefetch_4d(map, 64, head, t, bcoord);
    };

    constexpr uint32_t ID_P = ptx::idesc_bf16(128, 64, 0, 0, 0);
    constexpr uint32_t ID_W = ptx::idesc_bf16(128, 128, 1, 0, 0);
    constexpr uint32_t ID_U = ptx::idesc_bf16(128, 128, 1, 0, 0);
    constexpr uint32_t ID_WS = ptx::idesc_bf16(128, 128, 0, 1, 1);
    constexpr uint32_t ID_WS_HI = ptx::idesc_bf16(128, 64, 0, 1, 1);  // -S_lo^T W_hi^T
    constexpr uint32_t ID_O = ptx::idesc_bf16(128, 64, 0, 0, 0);
    constexpr uint32_t ID_S = ptx::idesc_bf16(128, 128, 0, 1, 0);
    // shared-memory descriptors (SW128, SBO 1024) by byte offset from sb, one per LBO
    const uint32_t dlo16 = ptx::sw128_desc_lo(sb, 16), dlo8k = ptx::sw128_desc_lo(sb, 8192),
                   dlo16k = ptx::sw128_desc_lo(sb, 16384);
    auto desc = [](uint32_t lo_base, uint32_t off) { return ptx::desc_pair(lo_base + (off >> 4), ptx::sw128_desc_hi(1024)); };

    auto aslot = [](int m) { return C_ASLOT + (uint32_t)(m % NSLOT) * ASLOT; };
    auto bslot = [](int m) { return C_BSLOT + (uint32_t)(m % NSLOT) * B_BYTES; };
    auto slot_par = [](int m) { return (uint32_t)((m / NSLOT) & 1); };
    if (compute) {
        // ============================== warpgroups 0-1 ==============================
        ptx::setmaxnreg_inc<COMPUTE_REGS>();
        float S[64];  // chain: S[dk = 64 half + j][dv = row]
        auto store_state_operand = [&]() {
#pragma unroll
            for (int c2 = 0; c2 < 2; ++c2) {
                uint32_t hi[16], lo[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) split2x(S[32 * c2 + 2 * j], S[32 * c2 + 2 * j + 1], hi[j], lo[j]);
                ptx::tmem_st16(tl + T_SA_HI + 32 * half + 16 * c2, hi);
                ptx::tmem_st16(tl + T_SA_LO + 32 * half + 16 * c2, lo);
            }
        };
        if (outcta && tid == 0) {  // arm the o slots for the first two chunks
            for (int s = 0; s < 2 && s < NC; ++s) {
                ++(s ? armed_o1 : armed_o0);
                ptx::mbar_arrive_expect_tx(bar(B_FULLO + s), O_BYTES);
            }
        }
        ptx::tc_fence_before();
        ptx::cluster_sync();  // every CTA's barriers are initialised and the slots armed
        ptx::tc_fence_after();

        if (chain) {
            // ---------------- chain CTA: state, operands, output
            {   // initial state operand (after the cluster barrier: the prep CTAs need not wait for it)
                const size_t sbase = ((size_t)seq * p.HV + h) * HD * HD;
#pragma unroll
                for (int j = 0; j < 64; ++j) {
                    const int dk = 64 * half + j;
                    S[j] = phi_unit ? (dk == row ? 1.f : 0.f)
                                    : ((p.s0 != nullptr) ? p.s0[sbase + (size_t)dk * HD + row] : 0.f);
                }
                store_state_operand();
                ptx::tmem_wait_st();
                hand_off(B_SOP);
            }
            float* ecl = misc + M_C / 4;  // e^c of chunks with even / odd index
            // ---- o(m) = scale e^c o1 + o2 -> bf16 staging buffer (chunk parity). Staged transposed,
            //      o^T [128 dv][64 tok] with 128-byte rows in 16-byte chunks XOR-swizzled by (dv & 7):
            //      one thread writes its row half with four 16-byte stores. Runs at the top of chunk
            //      m + 1's iteration, under the wait for C12(m + 1), so that it is off the recurrence.
            // Returns false when the wait for the output CTA's hand-back of the buffer ran out: the
            // buffer's slot in the output CTA is then not armed, and o(m) must not be shipped.
            auto stage_output = [&](int m) -> bool {
                wait_bar(B_Y, (uint32_t)(m & 1));
                ptx::tc_fence_after();
                // the output CTA has handed back this buffer (its chunk m - 2)
                bool handed_back = true;
                if (m >= 2 && !ptx::mbar_wait_compact(bar(B_EMPTYO + (m & 1)), (uint32_t)(((m >> 1) - 1) & 1), WAIT_ITERS)) {
                    fail();
                    handed_back = false;
                }
                const float* ecm = ecl + (m & 1) * CS;
                const uint32_t ob = sb + C_OST + (uint32_t)(m & 1) * O_BYTES;
#pragma unroll 1
                for (int h2 = 0; h2 < 2; ++h2) {  // 16 columns at a time (registers: the state is live)
                    float v[16], v2[16];
                    ptx::tmem_ld16(tl + T_O + 32 * half + 16 * h2, v);
                    ptx::tmem_ld16(tl + T_O2 + 32 * half + 16 * h2, v2);
                    ptx::tmem_wait_ld();
                    if (h2 == 1) hand_off(B_OFREE);
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj) v[jj] = fmaf(p.scale * ecm[32 * half + 16 * h2 + jj], v[jj], v2[jj]);
#pragma unroll
                    for (int c = 0; c < 2; ++c)
                        st_shared_v4(ob + sw_chunk(row, 4 * half + 2 * h2 + c, 128), pack_bf16(v[8 * c], v[8 * c + 1]),
                                     pack_bf16(v[8 * c + 2], v[8 * c + 3]), pack_bf16(v[8 * c + 4], v[8 * c + 5]),
                                     pack_bf16(v[8 * c + 6], v[8 * c + 7]));
                }
                ptx::fence_proxy_async_smem();  // the staging buffer is read by a bulk copy
                return handed_back;
            };
            // after a barrier of warps 0-7 that follows stage_output(m): thread 0 ships o(m) if its own
            // wait for the buffer's hand-back succeeded (a copy into an unarmed slot of the output CTA
            // could still be in flight when the cluster exits)
            auto ship_output = [&](int m, bool handed_back) {
                if (tid == 0 && handed_back) {
                    const uint32_t dst = ptx::mapa(sb + U_OSLOT + (uint32_t)(m & 1) * O_BYTES, OUT_RANK);
                    const uint32_t fb = ptx::mapa(sb + U_MISC + M_BAR + 8u * (uint32_t)(B_FULLO + (m & 1)), OUT_RANK);
                    ptx::bulk_copy_s2cluster(dst, sb + C_OST + (uint32_t)(m & 1) * O_BYTES, O_BYTES, fb);
                }
            };
            for (int n = 0; n <= NC; ++n) {  // step NC only stages and ships the last chunk's output
                if (vote_abort()) break;
                const uint32_t ph = (uint32_t)(n & 1);
                const float* ecn = ecl + (n & 1) * CS;
                const bool o_ok = (n > 0) ? stage_output(n - 1) : false;
                if (n == NC) {
                    if (n > 0) {
                        csync();
                        ship_output(n - 1, o_ok);
                    }
                    break;
                }

                // ---- v_new hi/lo and (v_new e^{cL-c}) hi/lo -> TMEM A operands; keep e^c
                wait_mma(ph);
                if (!ptx::mbar_wait_compact(bar(B_FULLA + n % NSLOT), slot_par(n), WAIT_ITERS)) fail();  // decay factors landed
                {
                    const uint32_t sp = aslot(n);
                    const float* ed_s = reinterpret_cast<const float*>(smem + sp + A_ED);
                    // 16 columns at a time (the state is live in registers)
#pragma unroll 1
                    for (int hq = 0; hq < 2; ++hq) {
                        float v[16];
                        {
                            float v2[16];
                            ptx::tmem_ld16(tl + T_C12 + 32 * half + 16 * hq, v);
                            ptx::tmem_ld16(tl + T_C12 + 64 + 32 * half + 16 * hq, v2);
                            ptx::tmem_wait_ld();
#pragma unroll
                            for (int jj = 0; jj < 16; jj += 2)
                                f2_unpack(f2_add(f2_pack(v[jj], v[jj + 1]), f2_pack(v2[jj], v2[jj + 1])), v[jj], v[jj + 1]);
                        }
                        uint32_t vh[8], vl[8], ph_[8], pl[8];
#pragma unroll
                        for (int j4 = 0; j4 < 4; ++j4) {
                            const float4 e4 = ld4(ed_s + 32 * half + 16 * hq + 4 * j4);
                            const int j = 2 * j4;
                            float w0, w1, w2, w3;
                            f2_unpack(f2_mul(f2_pack(v[2 * j], v[2 * j + 1]), f2_pack(e4.x, e4.y)), w0, w1);
                            f2_unpack(f2_mul(f2_pack(v[2 * j + 2], v[2 * j + 3]), f2_pack(e4.z, e4.w)), w2, w3);
                            split2x(v[2 * j], v[2 * j + 1], vh[j], vl[j]);
                            split2x(v[2 * j + 2], v[2 * j + 3], vh[j + 1], vl[j + 1]);
                            split2x(w0, w1, ph_[j], pl[j]);
                            split2x(w2, w3, ph_[j + 1], pl[j + 1]);
                        }
                        // the previous chunk's v_new^T M^T and dS have read these columns (Y and X1 waited)
                        const uint32_t c0 = 16 * half + 8 * hq;
                        ptx::tmem_st8(tl + T_VN_HI + c0, vh);
                        ptx::tmem_st8(tl + T_VN_LO + c0, vl);
                        ptx::tmem_st8(tl + T_VP_HI + c0, ph_);
                        ptx::tmem_st8(tl + T_VP_LO + c0, pl);
                    }
                    if (tid < CS) ecl[(n & 1) * CS + tid] = reinterpret_cast<const float*>(smem + sp + A_EC)[tid];
                    ptx::tmem_wait_st();
                    hand_off(B_VNR);
                }
                csync();  // e^c copied for every thread; o(n - 1) staged
                if (n > 0) ship_output(n - 1, o_ok);

                // ---- S <- e^{cL} S + dS; the new S^T hi/lo operand (S^T q^T has read the old one)
                wait_bar(B_X1, ph);
                ptx::tc_fence_after();
                {
                    const float gam = ecn[CS - 1];
#pragma unroll
                    for (int c2 = 0; c2 < 2; ++c2) {
                        float v[32];
                        ptx::tmem_ld32(tl + T_S + 64 * half + 32 * c2, v);
                        ptx::tmem_wait_ld();
                        if (c2 == 1) hand_off(B_TSFREE);  // dS read: C12 of the next chunk may start
#pragma unroll
                        for (int j = 0; j < 32; j += 2)
                            f2_unpack(f2_fma(f2_pack(gam, gam), f2_pack(S[32 * c2 + j], S[32 * c2 + j + 1]),
                                             f2_pack(v[j], v[j + 1])),
                                      S[32 * c2 + j], S[32 * c2 + j + 1]);
                    }
                }
                wait_bar(B_X2, ph);  // S^T q^T has read the old state operand
                ptx::tc_fence_after();
                if (n + 1 < NC) {
                    store_state_operand();
                    ptx::tmem_wait_st();
                    hand_off(B_SOP);
                }

            }
            if (!*abort_flag) {
                // final state: at (seq, blockIdx.y) (= (seq, h) outside a segmented state pass), or,
                // in a segmented output pass, only the last segment's, at (batch row, h)
                float* sfp = p.sf + ((size_t)seq * gridDim.y + blockIdx.y) * HD * HD;
                if (kSeg && p.sf_last_only)
                    sfp = (seq % p.seg_per_seq == p.seg_per_seq - 1)
                              ? p.sf + ((size_t)(seq / p.seg_per_seq) * p.HV + h) * HD * HD : nullptr;
                if (phi_unit) {  // the map Phi is stored transposed, PhiT[k][i] = Phi[i][k] (k = row)
                    float4* dst = reinterpret_cast<float4*>(sfp + (size_t)row * HD + 64 * half);
#pragma unroll
                    for (int j = 0; j < 16; ++j) dst[j] = make_float4(S[4 * j], S[4 * j + 1], S[4 * j + 2], S[4 * j + 3]);
                } else if (sfp != nullptr) {
#pragma unroll
                    for (int j = 0; j < 64; ++j) sfp[(size_t)(64 * half + j) * HD + row] = S[j];
                }
            }
        } else if (!outcta) {
            // ---------------- prep CTA
            const int pi = (int)rank - (int)PREP_RANK0;  // owns chunks pi, pi + NP, ...
            float* Ls = reinterpret_cast<float*>(smem + P_L);
            if (tid == 0 && pi < NC) {
                load_q(pi);
                load_k(pi);
            }

            int k = 0;
            for (int n = pi; n < NC; n += NP, ++k) {
                const uint32_t stg = P_STG + (uint32_t)(k & 1) * SLOT;
                // c, beta, e^c, e^{cL-c} of this chunk, written by the gate warp
                const float* gs = reinterpret_cast<const float*>(smem + P_GATE + (uint32_t)(k & 1) * GSLOT);
                const float *c_s = gs, *beta_s = gs + CS, *ec_s = gs + 2 * CS;  // e^{cL-c} follows e^c
                float* X = reinterpret_cast<float*>(smem + stg + SL_W);  // inversion scratch (W area not yet written)
                const uint32_t ph = (uint32_t)(k & 1);
                // thread 0 has confirmed that staging[k & 1] was shipped and consumed; every
                // thread takes the same exit decision
                if (vote_abort()) break;

                wait_bar(B_Q, ph);
                wait_bar(B_K, ph);
                if (tid == 0 && !*abort_flag) {
                    ptx::tc_fence_after();
#pragma unroll
                    for (int s = 0; s < 8; ++s) {
                        const uint32_t koff = (uint32_t)(s >> 2) * 16384u + (uint32_t)(s & 3) * 32u;
                        const uint64_t a = desc(dlo16, P_QK + koff);
                        const uint64_t b = desc(dlo16, P_QK + 8192 + koff);
                        ptx::mma_bf16(tmem + T_P, a, b, ID_P, s > 0);
                    }
                    commit();
                }
                csync();
                wait_bar(B_GREADY + (k & 1), (uint32_t)((k >> 1) & 1));  // gates (L, M need them; P1 does not)
                wait_mma(0u);  // P1: the CTA's commits alternate P1 (even phases) and P3 (odd)
                if (tid == 0 && !*abort_flag && n + NP < NC) load_q(n + NP);  // P1 has read q
                {   // rows 0-63: M = scale (q_i k_j) e^{c_i - c_j}, j <= i (hi/lo -> staging);
                    // rows 64-127: L = beta_i (k_i k_j) e^{c_i - c_j}, j < i (fp32 scratch).
                    // One loop for both, so that the loop body's code stays small.
                    float v[32];
                    ptx::tmem_ld32(tl + T_P + 32 * half, v);
                    ptx::tmem_wait_ld();
                    const bool mrow = row < CS;
                    const int i = mrow ? row : row - CS;
                    const float ci = c_s[i];
                    const float mul = mrow ? p.scale : beta_s[i];
                    const int jmax = mrow ? i : i - 1;  // last column kept
#pragma unroll
                    for (int j4 = 0; j4 < 8; ++j4) {
                        const float4 c4 = ld4(c_s + 32 * half + 4 * j4);
                        const float cj[4] = {c4.x, c4.y, c4.z, c4.w};
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const int jj = 4 * j4 + u, j = 32 * half + jj;
                            v[jj] = (j <= jmax) ? mul * v[jj] * ex2f((ci - cj[u]) * LOG2E) : 0.f;
                        }
                    }
                    if (mrow) {
#pragma unroll
                        for (int ch = 0; ch < 4; ++ch) {
                            const uint32_t co = sw_chunk(i, 4 * half + ch, 64);
                            put8_split(sb + stg + SL_M + co, sb + stg + SL_M + 8192 + co, v + 8 * ch, true);
                        }
                    } else {
                        float* lrow = Ls + i * LSTRIDE + 32 * half;
#pragma unroll
                        for (int j4 = 0; j4 < 8; ++j4)
                            *reinterpret_cast<float4*>(lrow + 4 * j4) =
                                make_float4(v[4 * j4], v[4 * j4 + 1], v[4 * j4 + 2], v[4 * j4 + 3]);
                    }
                }
                ptx::tc_fence_before();
                csync();
                invert_unit_lower<false>(Ls, X, tid, [](int) {}, csync);
                {   // T' -> staging (stacked hi/lo), T'' -> local
                    const int i = tid >> 2, jb = tid & 3;
                    float tp[16], tpp[16];
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) {  // T' = T diag(beta), T'' = T' diag(e^c), two columns per step
                        const float4 t4 = ld4(Ls + i * LSTRIDE + 16 * jb + 4 * q4);
                        const float4 b4 = ld4(beta_s + 16 * jb + 4 * q4), e4 = ld4(ec_s + 16 * jb + 4 * q4);
                        const int jj = 4 * q4;
                        const uint64_t p0 = f2_mul(f2_pack(t4.x, t4.y), f2_pack(b4.x, b4.y));
                        const uint64_t p1 = f2_mul(f2_pack(t4.z, t4.w), f2_pack(b4.z, b4.w));
                        f2_unpack(p0, tp[jj], tp[jj + 1]);
                        f2_unpack(p1, tp[jj + 2], tp[jj + 3]);
                        f2_unpack(f2_mul(p0, f2_pack(e4.x, e4.y)), tpp[jj], tpp[jj + 1]);
                        f2_unpack(f2_mul(p1, f2_pack(e4.z, e4.w)), tpp[jj + 2], tpp[jj + 3]);
                    }
#pragma unroll
                    for (int hh = 0; hh < 2; ++hh) {
                        const uint32_t co = sw_chunk(i, 2 * jb + hh, 64);
                        put8_split(sb + stg + SL_TP + co, sb + stg + SL_TP + 8192 + co, tp + 8 * hh, true);
                        put8_split(sb + P_TPP + co, sb + P_TPP + 8192 + co, tpp + 8 * hh, true);
                    }
                    if (tid < 2 * CS)  // decay factors travel with part A of the slot
                        reinterpret_cast<float*>(smem + stg + SL_EC)[tid] = ec_s[tid];
                }
                ptx::fence_proxy_async_smem();
                csync();
                if (tid == 0) ptx::mbar_arrive(bar(B_GFREE + (k & 1)));  // gate slot read
                if (tid == 0 && !*abort_flag) {  // P3: W^T = K^T [T''_hi; T''_lo]^T
                    ptx::tc_fence_after();
#pragma unroll
                    for (int s = 0; s < 4; ++s) {
                        const uint64_t a = desc(dlo16k, P_QK + 8192 + s * 2048);
                        const uint64_t b = desc(dlo16, P_TPP + s * 32);
                        ptx::mma_bf16(tmem + T_W, a, b, ID_W, s > 0);
                    }
                    commit();
                }
                wait_mma(1u);  // P3
                if (tid == 0 && !*abort_flag && n + NP < NC) {  // k consumed: fetch this CTA's next chunk
                    load_k(n + NP);
                    prefetch_tile(&p.tm_q, hq, n + 2 * NP);
                    prefetch_tile(&p.tm_k, hq, n + 2 * NP);
                }
                {   // W^T rows (dk = row) -> staging, hi and lo tiles 16 KB apart
                    float v[32], v2[32];
                    ptx::tmem_ld32(tl + T_W + 32 * half, v);
                    ptx::tmem_ld32(tl + T_W + 64 + 32 * half, v2);
                    ptx::tmem_wait_ld();
#pragma unroll
                    for (int jj = 0; jj < 32; jj += 2)
                        f2_unpack(f2_add(f2_pack(v[jj], v[jj + 1]), f2_pack(v2[jj], v2[jj + 1])), v[jj], v[jj + 1]);
#pragma unroll
                    for (int ch = 0; ch < 4; ++ch) {
                        const uint32_t co = sw_chunk(row, 4 * half + ch, 128);
                        put8_split(sb + stg + SL_W + co, sb + stg + SL_W + 16384 + co, v + 8 * ch, true);
                    }
                }
                ptx::tc_fence_before();
                ptx::fence_proxy_async_smem();
                csync();
                if (tid == 0 && !*abort_flag) {  // ship each part once the chain has handed back that part of the previous chunk
                    // A part is shipped only if its hand-back arrived: after a wait that ran out, the chain's
                    // slot is not armed, and the copy could still be in flight when the cluster exits.
                    auto wait_empty = [&](int b) { return !*abort_flag && wait_bar(b, (uint32_t)((k - 1) & 1)); };
                    // the chain CTA's slots and barriers sit at its own offsets, in CTA CHAIN_RANK
                    const uint32_t fa = ptx::mapa(sb + C_MISC + M_BAR + 8u * (uint32_t)(B_FULLA + pi), CHAIN_RANK);
                    const uint32_t fbb = ptx::mapa(sb + C_MISC + M_BAR + 8u * (uint32_t)(B_FULLB + pi), CHAIN_RANK);
                    const uint32_t da = ptx::mapa(sb + C_ASLOT + (uint32_t)pi * ASLOT, CHAIN_RANK);
                    const uint32_t db = ptx::mapa(sb + C_BSLOT + (uint32_t)pi * B_BYTES, CHAIN_RANK);
                    if (k == 0 || wait_empty(B_EMPTYA)) {
                        ptx::bulk_copy_s2cluster(da + A_TP, sb + stg + SL_TP, SL_M - SL_TP, fa);
                        ptx::bulk_copy_s2cluster(da + A_EC, sb + stg + SL_EC, 512, fa);
                    }
                    if (k == 0 || wait_empty(B_EMPTYB)) ptx::bulk_copy_s2cluster(db, sb + stg + SL_M, B_BYTES, fbb);
                }
            }
            if (tid == 0 && k >= 1 && !*abort_flag) {  // the last shipment must land before this CTA exits
#pragma unroll
                for (int b = B_EMPTYA; b <= B_EMPTYB; ++b) {
                    if (!ptx::mbar_wait_compact(bar(b), (uint32_t)((k - 1) & 1), WAIT_ITERS)) fail();
                }
            }
        } else {
            // ---------------- output CTA: gated-RMSNorm epilogue of every chunk (4 threads per
            // token, 16-byte chunks {eq, eq+4, eq+8, eq+12}); o arrives from the chain CTA, the gate
            // tile w * silu(z) from the gate warps (warpgroup 2), a chunk or two ahead
            const int et = tid >> 2, eq = tid & 3;
            for (int n = 0; n < NC; ++n) {
                if (vote_abort()) break;
                const int valid = min(CS, len - n * CS);
                const long long tok0 = tok_base + (long long)n * CS;
                const uint32_t par = (uint32_t)((n >> 1) & 1);
                const uint32_t oslot = U_OSLOT + (uint32_t)(n & 1) * O_BYTES;
                const uint32_t gate = U_GATE + (uint32_t)(n & 1) * GATE_BYTES;
                wait_bar(B_FULLO + (n & 1), par);
                {   // o^T -> o: thread (dv, token half) reads four 16-byte chunks of row dv
                    const int dv = tid >> 1, th = tid & 1;
                    __nv_bfloat16* ot = reinterpret_cast<__nv_bfloat16*>(smem + U_OT);
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        uint32_t w4[4];
                        ld_shared_v4(sb + oslot + sw_chunk(dv, 4 * th + c, 128), w4[0], w4[1], w4[2], w4[3]);
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const __nv_bfloat162 b2 = *reinterpret_cast<const __nv_bfloat162*>(&w4[u]);
                            const int t = 32 * th + 8 * c + 2 * u;
                            ot[sw_off(t, dv, 64) >> 1] = b2.x;
                            ot[sw_off(t + 1, dv, 64) >> 1] = b2.y;
                        }
                    }
                }
                csync();  // o slot read, o staged
                if (tid == 0 && !*abort_flag) {  // (after a failed wait the slot's phase may be pending: not re-armed)
                    if (n + 2 < NC) {  // this parity's slot takes chunk n + 2
                        if (n & 1) ++armed_o1;
                        else ++armed_o0;
                        ptx::mbar_arrive_expect_tx(bar(B_FULLO + (n & 1)), O_BYTES);
                    }
                    // the chain CTA's barriers sit at its own misc offset
                    ptx::mbar_arrive_remote(ptx::mapa(sb + C_MISC + M_BAR + 8u * (uint32_t)(B_EMPTYO + (n & 1)), CHAIN_RANK));
                }
                float o[32];
#pragma unroll
                for (int m = 0; m < 4; ++m) {
                    uint32_t w4[4];
                    ld_shared_v4(sb + U_OT + sw_chunk(et, eq + 4 * m, 64), w4[0], w4[1], w4[2], w4[3]);
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
                    wait_bar(B_OGFULL + (n & 1), par);  // this chunk's gate tile
                    float ss = 0.f;
#pragma unroll
                    for (int j = 0; j < 32; ++j) ss = fmaf(o[j], o[j], ss);
                    ss += __shfl_xor_sync(0xffffffffu, ss, 1);
                    ss += __shfl_xor_sync(0xffffffffu, ss, 2);
                    const float rstd = rsqrtf(ss * (1.f / (float)HD) + p.eps);
#pragma unroll
                    for (int m = 0; m < 4; ++m) {
                        const int c = eq + 4 * m;
                        const float4 g0 = *reinterpret_cast<const float4*>(smem + gate + gate_chunk(et, 2 * c));
                        const float4 g1 = *reinterpret_cast<const float4*>(smem + gate + gate_chunk(et, 2 * c + 1));
                        const float gg[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const int j = 8 * m + 2 * u;
                            outw[4 * m + u] = pack_bf16(bf16r(o[j] * rstd) * gg[2 * u], bf16r(o[j + 1] * rstd) * gg[2 * u + 1]);
                        }
                    }
                }
                if (et < valid && (!kSeg || p.out != nullptr)) {  // (a segmented state pass stores no output)
                    uint4* dst = reinterpret_cast<uint4*>(p.out + (size_t)(tok0 + et) * p.HV * HD + (size_t)h * HD);
#pragma unroll
                    for (int m = 0; m < 4; ++m)
                        dst[eq + 4 * m] = make_uint4(outw[4 * m], outw[4 * m + 1], outw[4 * m + 2], outw[4 * m + 3]);
                }
                csync();  // o tile and gate tile read
                if (tid == 0 && p.gated) ptx::mbar_arrive(bar(B_OGFREE + (n & 1)));  // the gate warps may refill it
            }
            // Abort path: wait (bounded) for the chain's o copies armed here
            if (*abort_flag && tid == 0) {
                drain(B_FULLO, armed_o0);
                drain(B_FULLO + 1, armed_o1);
            }
        }
        // Abort path: wait (bounded) for the TMA loads and MMAs this thread issued before
        // the shared memory and TMEM are released.
        if (*abort_flag && tid == 0 && !chain && !outcta) {  // prep: q / k tiles, P1 / P3
            drain(B_Q, armed_q);
            drain(B_K, armed_k);
            drain_mma(B_DRAIN);
        }
        csync();
        if (tid == 0) *done_flag = 1;  // lets the idle warps of warpgroup 2 stop sleeping
    } else {
        // ============================== warpgroup 2 ==============================
        ptx::setmaxnreg_dec<ISSUE_REGS>();
        const bool mma_warp = chain && warp == ISSUER_WARP;
        const bool producer = chain && warp == ISSUER_WARP + 1;
        const bool mma_out = chain && warp == ISSUER_WARP + 2;
        const bool gate_warp = !chain && !outcta && warp == ISSUER_WARP;
        const bool out_gate = outcta && p.gated;  // warpgroup 2 of the output CTA forms the gate tiles
        auto prep_bar = [&](int b, int m) {  // the prep CTAs' barriers sit at their own misc offset
            return ptx::mapa(sb + P_MISC + M_BAR + 8u * (uint32_t)b, (uint32_t)(PREP_RANK0 + m % NSLOT));
        };
        auto arm_slot = [&](int b, int m, uint32_t bytes) {
            const bool odd = (m % NSLOT) != 0;
            if (b == B_FULLA) ++(odd ? armed_a1 : armed_a0);
            else ++(odd ? armed_b1 : armed_b0);
            ptx::mbar_arrive_expect_tx(bar(b + m % NSLOT), bytes);
        };
        if (producer && lane == 0) {  // arm the slots for each prep CTA's first chunk
            for (int s = 0; s < NSLOT && s < NC; ++s) {
                arm_slot(B_FULLA, s, A_BYTES);
                arm_slot(B_FULLB, s, B_BYTES);
            }
        }
        __syncwarp();
        ptx::tc_fence_before();
        ptx::cluster_sync();  // every CTA's barriers are initialised and the slots armed
        ptx::tc_fence_after();

        if (mma_warp) {
            // ---------------- MMA issue. tcgen05.mma occupies the issuing thread for about the
            // instruction's execution time, so this warp issues MMAs and waits only on what
            // gates them; loads and slot hand-backs run on the producer warp.
            // A failed wait ends the loop: no MMA is issued on a tile or operand that did not arrive.
            if (lane == 0) {
                for (int n = 0; n < NC; ++n) {
                    if (*abort_flag) break;
                    const uint32_t ph = (uint32_t)(n & 1);
                    const uint32_t sp = aslot(n);
                    // ---- C12: v_new^T = v^T [T'_hi;T'_lo]^T - S^T [W_hi|W_lo] (hi terms cols 0-63, lo 64-127);
                    //      the v^T T'^T part does not depend on the state and goes first
                    if (!wait_bar(B_FULLA + n % NSLOT, slot_par(n)) || !wait_bar(B_V, ph)) break;
                    if (n > 0 && !wait_bar(B_TSFREE, (uint32_t)((n - 1) & 1))) break;  // dS of chunk n-1 read
                    ptx::tc_fence_after();
#pragma unroll
                    for (int s = 0; s < 4; ++s) {
                        const uint64_t a = desc(dlo8k, C_V + s * 2048);
                        const uint64_t b = desc(dlo16, sp + A_TP + s * 32);
                        ptx::mma_bf16(tmem + T_C12, a, b, ID_U, s > 0);
                    }
                    commit_to(B_VT);      // the v tile is free once these have run
                    if (!wait_bar(B_SOP, ph)) break;  // S_n^T hi/lo in TMEM
                    ptx::tc_fence_after();
#pragma unroll 1
                    for (int part = 0; part < 2; ++part) {
                        // S_hi [W_hi | W_lo], then S_lo W_hi (N = 64: the S_lo W_lo term is below
                        // the precision of the split and is left out)
                        const uint32_t sa = part ? T_SA_LO : T_SA_HI;
                        const uint32_t idw = part ? ID_WS_HI : ID_WS;
#pragma unroll
                        for (int s = 0; s < 8; ++s) {
                            const uint64_t b = desc(dlo16k, sp + A_W + s * 2048);
                            ptx::mma_bf16_ts(tmem + T_C12, tmem + sa + 8 * s, b, idw, 1u);
                        }
                    }
                    commit();
                    // ---- dS^T = (v_new e^{cL-c})^T K, once v_new is in TMEM
                    if (!wait_bar(B_K, ph) || !wait_bar(B_VNR, ph)) break;
                    ptx::tc_fence_after();
#pragma unroll 1
                    for (int part = 0; part < 2; ++part) {
                        const uint32_t va = part ? T_VP_LO : T_VP_HI;
#pragma unroll
                        for (int s = 0; s < 4; ++s) {
                            const uint64_t b = desc(dlo16k, C_QK + 8192 + s * 2048);
                            ptx::mma_bf16_ts(tmem + T_S, tmem + va + 8 * s, b, ID_S, (part | s) > 0);
                        }
                    }
                    commit_to(B_X1);
                }
                if (*abort_flag) drain_mma(B_DRAIN);  // every MMA this thread issued
            }
            __syncwarp();
        } else if (mma_out) {
            // ---------------- MMA issue for the output terms, off the state recurrence: S^T q^T
            // while warps 0-7 form v_new (after C12), v_new^T M^T while they update the state
            // (after dS), so that their issue time does not delay C12 and dS on warp 8.
            if (lane == 0) {  // a failed wait ends the loop, as on warp 8
                for (int n = 0; n < NC; ++n) {
                    if (*abort_flag) break;
                    const uint32_t ph = (uint32_t)(n & 1);
                    // ---- o1^T = S^T q^T, once the previous chunk's output accumulators are read
                    if (!wait_bar(B_MMA, ph) || !wait_bar(B_Q, ph)) break;  // C12 done: the tensor core is free
                    if (n > 0 && !wait_bar(B_OFREE, (uint32_t)((n - 1) & 1))) break;
                    ptx::tc_fence_after();
#pragma unroll 1
                    for (int part = 0; part < 2; ++part) {
                        const uint32_t sa = part ? T_SA_LO : T_SA_HI;
#pragma unroll
                        for (int s = 0; s < 8; ++s) {
                            const uint64_t b = desc(dlo16, C_QK + (s >> 2) * 16384 + (s & 3) * 32);
                            ptx::mma_bf16_ts(tmem + T_O, tmem + sa + 8 * s, b, ID_O, (part | s) > 0);
                        }
                    }
                    commit_to(B_X2);
                    // ---- o2^T = v_new^T M^T, once dS is done
                    if (!wait_bar(B_X1, ph) || !wait_bar(B_VNR, ph) || !wait_bar(B_FULLB + n % NSLOT, slot_par(n))) break;
                    ptx::tc_fence_after();
                    const uint32_t bp = bslot(n);
#pragma unroll 1
                    for (int term = 0; term < 3; ++term) {
                        const uint32_t va = (term == 1) ? T_VN_LO : T_VN_HI;
                        const uint32_t mb = bp + ((term == 2) ? 8192u : 0u);
#pragma unroll
                        for (int s = 0; s < 4; ++s) {
                            const uint64_t b = desc(dlo16, mb + s * 32);
                            ptx::mma_bf16_ts(tmem + T_O2, tmem + va + 8 * s, b, ID_O, (term | s) > 0);
                        }
                    }
                    commit_to(B_Y);
                }
                if (*abort_flag) drain_mma(B_DRAIN2);  // every MMA this thread issued
            }
            __syncwarp();
        } else if (producer) {
            // ---------------- TMA loads and slot hand-backs, each as soon as its buffer is free
            if (lane == 0 && NC > 0) {
                load_q(0);
                load_k(0);
                if (p.withhold_v_chunk != 0) load_v(0);
                // A failed wait ends the loop, and so does a failure of warps 0-7 (their flag is
                // released by the hand-off arrival this warp has just acquired): no tile is loaded
                // and no slot is re-armed while its previous phase may be pending.
                for (int n = 0; n < NC; ++n) {
                    if (*abort_flag) break;
                    const uint32_t ph = (uint32_t)(n & 1);
                    if (!wait_bar(B_VT, ph)) break;  // v^T T'^T has read the v tile
                    if (n + 1 < NC && n + 1 != p.withhold_v_chunk) load_v(n + 1);
                    if (!phi_unit) prefetch_tile(&p.tm_v, h, n + 2);
                    if (!wait_bar(B_VNR, ph) || *abort_flag) break;  // C12 read part A; decay factors copied
                    if (n + NSLOT < NC) arm_slot(B_FULLA, n, A_BYTES);
                    ptx::mbar_arrive_remote(prep_bar(B_EMPTYA, n));
                    if (!wait_bar(B_X1, ph) || !wait_bar(B_X2, ph)) break;  // dS, S^T q^T done: k, q tiles free
                    if (n + 1 < NC) {
                        load_q(n + 1);
                        load_k(n + 1);
                    }
                    prefetch_tile(&p.tm_q, hq, n + 2);
                    prefetch_tile(&p.tm_k, hq, n + 2);
                    if (!wait_bar(B_Y, ph)) break;  // v_new^T M^T done: part B free
                    if (n + NSLOT < NC) arm_slot(B_FULLB, n, B_BYTES);
                    ptx::mbar_arrive_remote(prep_bar(B_EMPTYB, n));
                }
                if (*abort_flag) {  // the TMA tiles and slot fills this thread armed
                    drain(B_Q, armed_q);
                    drain(B_K, armed_k);
                    drain(B_V, armed_v);
                    drain(B_FULLA, armed_a0);
                    drain(B_FULLA + 1, armed_a1);
                    drain(B_FULLB, armed_b0);
                    drain(B_FULLB + 1, armed_b1);
                }
            }
            __syncwarp();
        } else if (gate_warp) {
            // ---------------- prep CTA: in-chunk cumulative log-decay c (warp scan, lane l holds
            // tokens 2l and 2l+1), beta, e^c and e^{cL-c} of this CTA's chunks, up to two chunks
            // ahead of warps 0-7, so that none of it (global loads included) is on their path.
            const int pi = (int)rank - (int)PREP_RANK0;
            int k = 0;
            for (int n = pi; n < NC; n += NP, ++k) {
                if (__any_sync(0xffffffffu, *abort_flag != 0)) break;  // one decision for the warp (shuffles below)
                if (k >= 2) wait_bar(B_GFREE + (k & 1), (uint32_t)(((k >> 1) - 1) & 1));
                const int valid = min(CS, len - n * CS);
                const long long t0 = tok_base + (long long)n * CS;
                float g0 = 0.f, g1 = 0.f, b0 = 0.f, b1 = 0.f;
                if (2 * lane < valid) {
                    g0 = __ldg(p.g + (size_t)(t0 + 2 * lane) * p.HV + h);
                    b0 = __ldg(p.beta + (size_t)(t0 + 2 * lane) * p.HV + h);
                }
                if (2 * lane + 1 < valid) {
                    g1 = __ldg(p.g + (size_t)(t0 + 2 * lane + 1) * p.HV + h);
                    b1 = __ldg(p.beta + (size_t)(t0 + 2 * lane + 1) * p.HV + h);
                }
                float sc = g0 + g1;
#pragma unroll
                for (int off = 1; off < 32; off <<= 1) {
                    const float t = __shfl_up_sync(0xffffffffu, sc, off);
                    if (lane >= off) sc += t;
                }
                const float c1 = sc, c0 = sc - g1;
                const float cL = __shfl_sync(0xffffffffu, c1, 31);
                float* gs = reinterpret_cast<float*>(smem + P_GATE + (uint32_t)(k & 1) * GSLOT);
                gs[2 * lane] = c0;
                gs[2 * lane + 1] = c1;
                gs[CS + 2 * lane] = b0;
                gs[CS + 2 * lane + 1] = b1;
                gs[2 * CS + 2 * lane] = ex2f(c0 * LOG2E);
                gs[2 * CS + 2 * lane + 1] = ex2f(c1 * LOG2E);
                gs[3 * CS + 2 * lane] = ex2f((cL - c0) * LOG2E);
                gs[3 * CS + 2 * lane + 1] = ex2f((cL - c1) * LOG2E);
                ptx::mbar_arrive(bar(B_GREADY + (k & 1)));  // every lane: its stores are released
            }
            __syncwarp();
        } else if (out_gate) {
            // ---------------- output CTA, warpgroup 2: the gate tile w * silu(z) of every chunk (SFU-bound)
            // into one of two tiles (chunk parity), up to two chunks ahead of warps 0-7, which then run
            // only the transpose and the norm. Thread 256 issues the z loads (two tiles, chunk parity).
            const int gt = tid - ISSUER_WARP * 32;  // 0..127
            auto gsync = [] { ptx::named_sync(GSYNC, 128); };
            auto load_zt = [&](int n) {
                if (n & 1) load_tile(B_ZT + 1, U_Z + O_BYTES, &p.tm_z, h, n, armed_z1);
                else load_tile(B_ZT, U_Z, &p.tm_z, h, n, armed_z0);
            };
            w_s[gt] = __bfloat162float(p.w[gt]);
            if (gt == 0)
                for (int s = 0; s < 2 && s < NC; ++s) load_zt(s);
            gsync();  // w_s visible to the four warps
            for (int n = 0; n < NC; ++n) {
                if (ptx::named_sync_or(GSYNC, 128, *abort_flag != 0)) break;  // one decision for the four warps
                const uint32_t par = (uint32_t)((n >> 1) & 1);
                // the tile was read by chunk n-2's epilogue, and z(n) has landed (a failed wait skips the
                // work but not the barrier below, which every thread of the four warps reaches)
                bool ok = n < 2 || wait_bar(B_OGFREE + (n & 1), (uint32_t)(((n >> 1) - 1) & 1));
                ok = ok && wait_bar(B_ZT + (n & 1), par);
                const uint32_t zt = U_Z + (uint32_t)(n & 1) * O_BYTES;
                const uint32_t gate = U_GATE + (uint32_t)(n & 1) * GATE_BYTES;
                for (int u = gt; ok && u < CS * 16; u += 128) {
                    const int r = u >> 4, zc = u & 15;
                    uint32_t w4[4];
                    ld_shared_v4(sb + zt + sw_chunk(r, zc, 64), w4[0], w4[1], w4[2], w4[3]);
                    float gv[8];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const __nv_bfloat162 z2 = *reinterpret_cast<const __nv_bfloat162*>(&w4[e]);
                        const float z0 = __low2float(z2), z1 = __high2float(z2);
                        gv[2 * e] = w_s[8 * zc + 2 * e] * (z0 * rcpf(1.f + ex2f(-z0 * LOG2E)));
                        gv[2 * e + 1] = w_s[8 * zc + 2 * e + 1] * (z1 * rcpf(1.f + ex2f(-z1 * LOG2E)));
                    }
                    *reinterpret_cast<float4*>(smem + gate + gate_chunk(r, 2 * zc)) = make_float4(gv[0], gv[1], gv[2], gv[3]);
                    *reinterpret_cast<float4*>(smem + gate + gate_chunk(r, 2 * zc + 1)) = make_float4(gv[4], gv[5], gv[6], gv[7]);
                }
                gsync();  // the gate tile is written and the z tile read by all four warps
                if (gt == 0 && !*abort_flag) {
                    ptx::mbar_arrive(bar(B_OGFULL + (n & 1)));  // (after the barrier: every gate store precedes it)
                    if (n + 2 < NC) {                        // this parity's z tile takes chunk n + 2
                        ptx::fence_proxy_async_smem();
                        load_zt(n + 2);
                        prefetch_tile(&p.tm_z, h, n + 3);
                    }
                }
            }
            if (gt == 0 && *abort_flag) {  // the z loads this thread armed, before the CTA leaves
                drain(B_ZT, armed_z0);
                drain(B_ZT + 1, armed_z1);
            }
            __syncwarp();
        } else {
            // Idle warps sleep until warps 0-7 are done instead of waiting at the cluster
            // barrier for the whole kernel, where they would take issue slots from the
            // working warps of this SM. Bounded; the barrier below is what synchronises.
            if (lane == 0)
                for (uint32_t it = 0; it < (1u << 21) && *done_flag == 0; ++it) __nanosleep(1000);
            __syncwarp();
        }
    }
    ptx::tc_fence_before();
    ptx::cluster_sync();  // no CTA leaves while a peer may still touch its shared memory
    if (warp == 0 && tmem_cols > 0) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem, tmem_cols);
    }
}

}  // namespace split

// The kernel's register split (setmaxnreg) assumes exactly LAUNCH_REGS registers per
// thread at launch; with fewer, the increase in warpgroups 0-1 would never be granted.
// The compiled count is checked once per device and the kernel is not launched unless
// it matches.
static cudaError_t split_prepare(int dev) {
    // 0 unchecked, 1 ready, 2 unusable; threads that race here do the same idempotent checks
    static std::atomic<int> state[64] = {};
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (state[dev].load(std::memory_order_acquire) == 0) {
        int ok = 1;
        for (auto fn : {split::gdn_prefill_split_kernel<false>, split::gdn_prefill_split_kernel<true>}) {
            cudaFuncAttributes fa;
            cudaError_t e = cudaFuncGetAttributes(&fa, fn);
            if (e != cudaSuccess) return e;
            if (fa.numRegs != split::LAUNCH_REGS) {
                ok = 0;
                break;
            }
            e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)split::SMEM_ALLOC);
            if (e != cudaSuccess) return e;
        }
        state[dev].store(ok ? 1 : 2, std::memory_order_release);
    }
    return state[dev].load(std::memory_order_acquire) == 1 ? cudaSuccess : cudaErrorNotSupported;
}

bool split_available() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    return split_prepare(dev) == cudaSuccess;
}

cudaError_t launch_split(const Params& p, int nseq, int grid_heads, cudaStream_t stream) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    e = split_prepare(dev);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(split::CLUSTER, grid_heads, nseq);
    cfg.blockDim = dim3(split::NTHREADS, 1, 1);
    cfg.dynamicSmemBytes = split::SMEM_ALLOC;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = split::CLUSTER;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    // programmatic dependent launch: the kernel waits for the previous grid before touching memory
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    e = p.seg_chunks > 0 ? cudaLaunchKernelEx(&cfg, split::gdn_prefill_split_kernel<true>, p)
                         : cudaLaunchKernelEx(&cfg, split::gdn_prefill_split_kernel<false>, p);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

int split_cluster_ctas() { return split::CLUSTER; }

// Clusters of the split kernel that fit the current device at once (one wave), from the
// occupancy API (clusters must fit inside a GPC, so this can be below SMs / cluster size;
// 32 on B200 against 148 / 4 = 37); 0 if the kernel cannot run. Cached per device.
int split_clusters_per_wave() {
    static std::atomic<int> cache[64] = {};  // 0 unknown, -1 no answer, else clusters per wave
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    if (cache[dev].load(std::memory_order_acquire) == 0) {
        if (split_prepare(dev) != cudaSuccess) return 0;
        cudaLaunchConfig_t cfg;
        memset(&cfg, 0, sizeof(cfg));
        cfg.gridDim = dim3(split::CLUSTER, 1, 1);
        cfg.blockDim = dim3(split::NTHREADS, 1, 1);
        cfg.dynamicSmemBytes = split::SMEM_ALLOC;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = split::CLUSTER;
        attr.val.clusterDim.y = 1;
        attr.val.clusterDim.z = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, split::gdn_prefill_split_kernel<false>, &cfg) != cudaSuccess) {
            cudaGetLastError();  // clear it: the caller falls back to SMs / cluster size
            n = -1;
        }
        cache[dev].store(n, std::memory_order_release);
    }
    const int n = cache[dev].load(std::memory_order_acquire);
    return n > 0 ? n : 0;
}

}  // namespace gdn
