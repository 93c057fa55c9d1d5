// Chunked gated-delta-rule (gated DeltaNet) prefill with a fused gated-RMSNorm
// epilogue, written for B200 (sm_100a): TMA-staged tiles, tcgen05 tensor-core
// MMAs with TMEM accumulators, and the recurrent state kept on chip.
//
// One CTA owns one (sequence, v-head) pair and walks its 64-token chunks in
// order. Per chunk n (c = in-chunk cumsum of g, L = strict-lower
// beta_i (k_i.k_j) e^{c_i-c_j}, T = (I+L)^-1):
//   --  gates: c, e^c, e^{c_L-c} by a warp scan (warp 1, while thread 0 issues P1)
//   P1  [Q;K] K^T            -> q.k (rows 0-63) and k.k (rows 64-127)  tcgen05, M=128
//   --  L, M = scale (q k^T) * decay  (registers); T: diagonal blocks by forward
//       substitution (CUDA cores), off-diagonal block products as tf32x3 mma.sync
//   P3  W^T  = K^T (T diag(beta e^c))^T, with C12's state-free part v^T T'^T  tcgen05, M=128
//   C12 v_new^T = v^T (T diag(beta))^T - S^T W^T  (in the dS columns) tcgen05, M=128
//   C4  dS^T = (v_new e^{c_L-c})^T K                                 tcgen05, M=128, N=128
//   C3  o^T  = scale e^c (S^T q^T) + v_new^T M^T  (two accumulators)  tcgen05, M=128
//   --  S <- e^{c_L} S + dS (fp32 registers) while C3 runs; o -> gated RMSNorm -> y
//   --  gate = w * silu(z) by every thread while C12 runs; read by the norm epilogue
// Thread 0 issues the MMAs but v_new^T M^T, which thread 32 issues once dS is in the
// tensor pipe (an issue occupies the thread for about the instruction's execution
// time); dS, S^T q^T and v_new^T M^T commit to separate barriers so that the state
// update and the new state operand overlap C3.
// Transposed forms put the 128-wide feature dimension on the MMA M axis so
// every accumulator row is one TMEM lane, which makes the state update
// thread-local; the norm epilogue re-reads o through a swizzled shared tile
// with four threads per token and 16-byte loads and stores.
//
// Precision: every operand that is not already a bf16 input (S, W, T', T'',
// v_new, M) is split into bf16 hi + lo parts, so products keep ~16 mantissa
// bits; accumulation is fp32 in TMEM; the state itself is fp32 in registers.
// The per-chunk operands S^T and v_new^T are written by their owning threads
// straight into TMEM and consumed there as the MMA A operand, which halves
// the shared-memory traffic of those MMAs.
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
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <mutex>

#include "gdn_common.cuh"
#include "gdn_prefill.h"
#include "sm100_ptx.cuh"

namespace gdn {

constexpr int NTHREADS = 256;  // 8 warps: warps w and w+4 share TMEM lane quarter w
constexpr uint32_t TMEM_COLS = 512;

// ---- shared-memory map (bytes from a 1024-aligned base) -------------------
// bf16 tiles use the 128-byte-swizzle layout TMA writes: a tile of R rows x
// 128 columns is two 64-column "panels" of R rows x 128 B; inside a panel the
// 16-byte chunk j of row r sits at chunk position j ^ (r & 7).
constexpr uint32_t OFF_QK = 0;           // panel p: q rows 0-63 | k rows 64-127 (16 KB/panel)
constexpr uint32_t OFF_V = 32768;        // v tile  [64 tok][128 dv]  (8 KB/panel)
constexpr uint32_t OFF_Z = 49152;        // z tile  [64 tok][128 dv]
constexpr uint32_t OFF_X = 65536;        // 64 KB: T', T'' (hi/lo), W (hi/lo); inversion scratch
constexpr uint32_t OFF_TP_HI = OFF_X + 0;       //  T'  = T diag(beta)        [64][64]
constexpr uint32_t OFF_TP_LO = OFF_X + 8192;
constexpr uint32_t OFF_TPP_HI = OFF_X + 16384;  //  T'' = T diag(beta e^c)    [64][64]
constexpr uint32_t OFF_TPP_LO = OFF_X + 24576;
constexpr uint32_t OFF_W_HI = OFF_X + 32768;    //  W^T [128 dk][64 tok] (MN-major B operand)
constexpr uint32_t OFF_W_LO = OFF_X + 49152;    //  (must follow W_HI by 16 KB: stacked along N)
constexpr uint32_t OFF_XTMP = OFF_X + 0;        //  inversion products (fp32, 4.5 KB)
constexpr uint32_t OFF_M_HI = 131072;    // M = scale (q k^T) * decay, [64][64] bf16
constexpr uint32_t OFF_M_LO = 139264;
constexpr uint32_t OFF_L = 147456;       // L / T fp32 [64][68]; o staging afterwards (8 KB/panel)
constexpr uint32_t OFF_OST = OFF_L;
constexpr uint32_t OFF_GATE = OFF_L + 64 * LSTRIDE * 4;  // 164864: w * silu(z), fp32 [64][128], 16-B chunks swizzled
constexpr uint32_t OFF_MISC = OFF_GATE + 32768;          // 197632
constexpr uint32_t MISC_C = 0;      // c        [64] f32
constexpr uint32_t MISC_BETA = 256; // beta     [64]
constexpr uint32_t MISC_EC = 512;   // e^c      [64]
constexpr uint32_t MISC_ED = 768;   // e^{cL-c} [64]
constexpr uint32_t MISC_BAR = 1024; // NBAR mbarriers
constexpr uint32_t MISC_TMEM = 1104;
constexpr uint32_t MISC_FLAG = 1108;
constexpr uint32_t MISC_W = 1152;   // norm weight [128] f32
constexpr uint32_t MISC_BYTES = 1664;
constexpr uint32_t SMEM_BYTES = OFF_MISC + MISC_BYTES;
// A record of the segmented passes' workspace: one chunk's T' hi/lo (the 16 KB at OFF_TP_HI) and
// W^T hi/lo (the 32 KB at OFF_W_HI), byte for byte.
constexpr uint32_t WREC_BYTES = 16384 + 32768;
static_assert(OFF_TP_LO == OFF_TP_HI + 8192 && OFF_W_LO == OFF_W_HI + 16384, "a record is two contiguous tiles");
constexpr uint32_t SMEM_ALLOC = SMEM_BYTES + 1024;  // slack for manual 1024 alignment
static_assert(SMEM_ALLOC <= 232448, "exceeds the 227 KB per-block shared memory limit");

// ---- TMEM map (columns; all 128 lanes). Regions are shared by operands
// whose lifetimes do not overlap within a chunk.
constexpr uint32_t TM_P = 0;       // P1 [Q;K]K^T fp32 (64)      -> then v_new^T hi/lo A operands
constexpr uint32_t TM_VN_HI = 0;   //   v_new^T bf16 pairs (32)
constexpr uint32_t TM_VN_LO = 32;
constexpr uint32_t TM_VP_HI = 64;  // (v_new e^{cL-c})^T hi/lo (64)
constexpr uint32_t TM_VP_LO = 96;
constexpr uint32_t TM_W = 128;     // P3 [T''_hi | T''_lo] parts of W^T fp32 (128), read before C12
constexpr uint32_t TM_O = 128;     // C3 S^T q^T (64)
constexpr uint32_t TM_O2 = 192;    //    v_new^T M^T (64)
constexpr uint32_t TM_S = 256;     // C12 [hi-part | lo-part] v_new^T fp32 (128), then C4 dS^T fp32 (128)
constexpr uint32_t TM_C12 = TM_S;
constexpr uint32_t TM_SA_HI = 384; // S^T bf16 pairs, A operand of C12 / C3 (64)
constexpr uint32_t TM_SA_LO = 448;

// Barrier slots: TMA tiles; MMA commit groups (BAR_MMA: every group but the two below, which
// let the state update start while the output products still run: BAR_DS = dS, BAR_O1 = S^T q^T,
// BAR_O2 = v_new^T M^T, issued by thread 32 once thread 0 has issued dS and arrived on BAR_DSI).
enum { BAR_Q = 0, BAR_K = 1, BAR_V = 2, BAR_Z = 3, BAR_MMA = 4, BAR_DS = 5, BAR_O1 = 6, BAR_O2 = 7, BAR_DSI = 8,
       BAR_W = 9 /* segmented output pass: T' and W^T tiles from the state pass */, NBAR = 10 };
static_assert(MISC_BAR + 8 * NBAR <= MISC_TMEM, "barriers overlap the TMEM address word");


// Debug record layout (floats) per (seq, head, chunk).
constexpr int DBG_C = 0, DBG_T = 64, DBG_W = DBG_T + 4096, DBG_VN = DBG_W + 8192,
              DBG_O = DBG_VN + 8192, DBG_SC = DBG_O + 8192, DBG_REC = DBG_SC + 16384;

// The pre-stage (TRT adapter) mode and the debug dumps are template parameters: the
// instantiation that serves the plain and gated paths carries neither's code in its loop
// (the kernel is sensitive to instruction fetch; its loop body is larger than an SM's
// instruction cache). So are the passes of a segmented call (kSeg, below).
//
// The passes of a segmented call. Block z indexes (sequence b, segment j) = (z / seg_per_seq,
// z % seg_per_seq), covering tokens [j seg_chunks 64, min((j+1) seg_chunks 64, T)) of batch row b;
// grid y = HV. A record of wbuf holds the T' and W^T hi/lo tiles of one chunk of one (sequence,
// segment, head) as the zero-state run formed them (48 KB, the shared-memory tile layout), indexed
// by (b, j, head, chunk) with seg_total segments per sequence.
// kSeg = SEG_STATE: the zero-state runs of every segment: v-head y from a zero state (s0 null).
//   Stores every chunk's record, and (but the last segment) its final state A at [b (seg_total-1)
//   + j][y] of the [.][2 HV] map array sf. Nothing else is formed: no q load, no M, no output
//   products, no norm.
// kSeg = SEG_PHI: the identity runs of every segment but the last (seg_per_seq = seg_total - 1):
//   v-head y from the identity with v = 0. Its chunk update needs only W (from the record), k and
//   the gates, so it forms no chunk preparation (no P1, L, inverse, T', P3) and loads no q or v; k
//   alternates between the two halves of the [q; k] panels so that the next chunk's k loads a
//   chunk ahead. Writes its final state, the map Phi, transposed (the layout the entry-state scan
//   reads) at [z][HV + y] of sf.
// kSeg = SEG_OUTPUT: every segment from its entry state s0[z], with the full outputs; it forms M
//   (P1) but takes T' and W^T from the records (no L, inverse, T'/T'' split or P3). Only the last
//   segment of each sequence writes its final state, at sf[b].
constexpr int SEG_NONE = 0, SEG_OUTPUT = 1, SEG_STATE = 2, SEG_PHI = 3;

// A bounded wait that ran out: set the CTA's abort flag and record bits 0 and 15 (this kernel) in the
// status word. Out of line: it runs only after a timeout, and inlined at each wait site it would put
// cold code between the hot loop's instructions (the kernel is sensitive to instruction fetch).
__device__ __noinline__ void record_failure_fused(volatile int* abort_flag, unsigned int* status) {
    *abort_flag = 1;
    if (status) atomicOr(status, 1u | (1u << 15));
}
template <bool kPrestage, bool kDebug, int kSeg = SEG_NONE>
__global__ void __launch_bounds__(NTHREADS, 1) gdn_prefill_kernel(const __grid_constant__ Params p) {
    constexpr bool kState = (kSeg == SEG_STATE);
    constexpr bool kPhi = (kSeg == SEG_PHI);
    constexpr bool kLean = kState || kPhi;  // no q, M, output products or norm
    constexpr bool kPrepped = (kSeg == SEG_OUTPUT);  // T' and W^T from the zero-state runs' records
    // identity run (v = 0, identity entry state)
    constexpr bool phi_unit = kPhi;
    // the tensor maps are kernel parameters, not data of the previous launch: fetch them while it ends
    if (threadIdx.x == 0) {
        if (!kLean) ptx::prefetch_tensormap(&p.tm_q);
        ptx::prefetch_tensormap(&p.tm_k);
        if (!phi_unit) ptx::prefetch_tensormap(&p.tm_v);
        if (p.gated) ptx::prefetch_tensormap(&p.tm_z);
    }
    // inputs may come from the previous launch in the stream: nothing global is touched before this
    ptx::grid_dependency_wait();
    ptx::grid_launch_dependents();
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    const uint32_t sb = ptx::smem_u32(smem);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int quarter = warp & 3, half = warp >> 2;
    const int row = quarter * 32 + lane;  // TMEM lane of this thread for M=128 accumulators
    const int h = (int)blockIdx.y;
    const int seq = blockIdx.z;
    const int hq = h / (p.HV / p.HQK);

    int t_begin, len, bcoord;
    if (kSeg != SEG_NONE) {  // segment seq % seg_per_seq of batch row seq / seg_per_seq
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
        for (int i = 0; i < NBAR; ++i) ptx::mbar_init(bar(i), 1);
        ptx::fence_mbar_init();
        *abort_flag = 0;
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
    const uint32_t tl = tmem + lane_addr;

    // S^T hi/lo (bf16 pairs) into TMEM as the A operand of C12 / C3:
    // thread (dv = row, half) owns dk in [64*half, 64*half + 64) = 32 packed columns.
    float S[64];
    auto store_state_operand = [&]() {
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2) {
            uint32_t hi[16], lo[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) split2(S[32 * c2 + 2 * j], S[32 * c2 + 2 * j + 1], hi[j], lo[j]);
            ptx::tmem_st16(tl + TM_SA_HI + 32 * half + 16 * c2, hi);
            ptx::tmem_st16(tl + TM_SA_LO + 32 * half + 16 * c2, lo);
        }
    };
    {
        const size_t sbase = ((size_t)seq * p.HV + h) * HD * HD;
#pragma unroll
        for (int j = 0; j < 64; ++j) {
            const int dk = 64 * half + j;
            // plain load: the adapter passes the same buffer as s0 and sf (read here, written at exit)
            S[j] = phi_unit ? (dk == row ? 1.f : 0.f) : ((p.s0 != nullptr) ? p.s0[sbase + (size_t)dk * HD + row] : 0.f);
        }
        store_state_operand();
    }
    // Epilogue mapping: token et = tid / 4, 16-byte output chunks {eq, eq+4, eq+8, eq+12}.
    const int et = tid >> 2, eq = tid & 3;
    float* w_s = misc + MISC_W / 4;
    if (tid < HD)
        w_s[tid] = !p.gated ? 0.f
                   : (kPrestage ? __half2float(reinterpret_cast<const __half*>(p.w)[tid]) : __bfloat162float(p.w[tid]));

    // ---- TMA issue helpers (thread 0) ----
    uint32_t issued[NBAR] = {}, consumed[NBAR] = {};
    auto load_q = [&](int n) {
        ++issued[BAR_Q];
        ptx::mbar_arrive_expect_tx(bar(BAR_Q), 16384);
        const int t = t_begin + n * CS;
        ptx::tma_load_4d(sb + OFF_QK + 0, &p.tm_q, bar(BAR_Q), 0, hq, t, bcoord);
        ptx::tma_load_4d(sb + OFF_QK + 16384, &p.tm_q, bar(BAR_Q), 64, hq, t, bcoord);
    };
    // Offset of chunk n's k rows inside the [q; k] panels: rows 64-127; an identity-run pass
    // alternates between rows 64-127 (even chunks) and rows 0-63 (odd chunks).
    auto koff = [](int n) -> uint32_t { return (kPhi && (n & 1)) ? 0u : 8192u; };
    auto load_k = [&](int n) {
        ++issued[BAR_K];
        ptx::mbar_arrive_expect_tx(bar(BAR_K), 16384);
        const int t = t_begin + n * CS;
        ptx::tma_load_4d(sb + OFF_QK + koff(n), &p.tm_k, bar(BAR_K), 0, hq, t, bcoord);
        ptx::tma_load_4d(sb + OFF_QK + 16384 + koff(n), &p.tm_k, bar(BAR_K), 64, hq, t, bcoord);
    };
    // Chunk n's record in wbuf: T' hi/lo (16 KB) then W^T hi/lo (32 KB). The identity-run pass loads
    // W^T into two alternating shared-memory buffers (the T'/T'' area is free there; the v barrier
    // counts those loads); the output pass loads both into their own places (barrier W).
    const int seg_j = kSeg != SEG_NONE ? seq - bcoord * p.seg_per_seq : 0;
    auto wrec = [&](int n) -> size_t {
        return ((((size_t)bcoord * p.seg_total + seg_j) * p.HV + h) * p.seg_chunks + n) * WREC_BYTES;
    };
    auto wtile = [](int n) -> uint32_t { return (n & 1) ? OFF_X : OFF_W_HI; };
    auto load_w = [&](int n) {
        ++issued[BAR_V];
        ptx::mbar_arrive_expect_tx(bar(BAR_V), 32768);
        ptx::bulk_load_g2s(sb + wtile(n), p.wbuf + wrec(n) + 16384, 32768, bar(BAR_V));
    };
    auto load_tw = [&](int n) {
        ++issued[BAR_W];
        ptx::mbar_arrive_expect_tx(bar(BAR_W), WREC_BYTES);
        ptx::bulk_load_g2s(sb + OFF_TP_HI, p.wbuf + wrec(n), 16384, bar(BAR_W));
        ptx::bulk_load_g2s(sb + OFF_W_HI, p.wbuf + wrec(n) + 16384, 32768, bar(BAR_W));
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
    // A failure is recorded as bit 0 plus bit 15 (this kernel) of the status word. Loads are
    // issued only while no failure is recorded: after a failed wait the phase waited for may
    // still be pending, and a new load would arm it a second time.
    auto fail = [&]() { record_failure_fused(abort_flag, p.status); };
    auto wait_bar = [&](int i, uint32_t parity) {
        if (ptx::mbar_wait(bar(i), parity, WAIT_ITERS)) ++consumed[i];
        else fail();
    };
    auto wait_mma = [&]() {
        wait_bar(BAR_MMA, consumed[BAR_MMA] & 1u);
        ptx::tc_fence_after();
    };
    auto commit_to = [&](int b) {
        ptx::mma_commit(bar(b));
        ++issued[b];
    };
    auto commit = [&]() { commit_to(BAR_MMA); };

    if (tid == 0 && NC > 0) {
        if (!kLean) load_q(0);
        load_k(0);
        if (p.withhold_v_chunk != 0 && !phi_unit) load_v(0);
        if (kPhi) load_w(0);
        if (kPrepped) load_tw(0);
    }
    if (tid == 128 && NC > 0 && p.gated) load_z(0);  // z feeds the gate product (while C12 runs)
    // Gate inputs of the next chunk are prefetched into warp 1's registers (lane l: tokens 2l,
    // 2l+1) as raw values: loaded unconditionally (positions past the sequence end are clamped
    // to its last token), transformed and masked only when that chunk is processed, so that
    // nothing waits on these loads earlier.
    float gn0 = 0.f, gn1 = 0.f, bn0 = 0.f, bn1 = 0.f;         // g, beta
    __half an0 = __float2half(0.f), an1 = an0, bh0 = an0, bh1 = an0;  // pre-stage a, b
    // Pre-stage gate math (gdnChunkPrefillSm87.cu:44-49, 113-125):
    // g = -exp(A_log[h]) * softplus(a + dt_bias[h]) (threshold 20), beta = sigmoid(b).
    const float gA = kPrestage ? -expf(__ldg(p.A_log + h)) : 0.f;
    const float gdt = kPrestage ? __half2float(p.dt_bias[h]) : 0.f;
    auto load_gates = [&](int n) {
        const int last = len - n * CS - 1;
        const long long t0 = tok_base + (long long)n * CS;
        const size_t i0 = (size_t)(t0 + min(2 * lane, last)) * p.HV + h;
        const size_t i1 = (size_t)(t0 + min(2 * lane + 1, last)) * p.HV + h;
        if (kPrestage) {
            an0 = ldg_early(p.ga + i0);
            bh0 = ldg_early(p.gb + i0);
            an1 = ldg_early(p.ga + i1);
            bh1 = ldg_early(p.gb + i1);
        } else {
            gn0 = ldg_early(p.g + i0);
            bn0 = ldg_early(p.beta + i0);
            gn1 = ldg_early(p.g + i1);
            bn1 = ldg_early(p.beta + i1);
        }
    };
    auto gate_of = [&](bool valid, float g_raw, float b_raw, __half a_raw, __half bb_raw, float& gv, float& bv) {
        if (!valid) {
            gv = bv = 0.f;
        } else if (kPrestage) {
            const float x = __half2float(a_raw) + gdt;
            gv = gA * (x > 20.f ? x : log1pf(expf(x)));
            bv = 1.f / (1.f + expf(-__half2float(bb_raw)));
        } else {
            gv = g_raw;
            bv = b_raw;
        }
    };
    if (warp == 1 && NC > 0) load_gates(0);
    ptx::tmem_wait_st();
    ptx::tc_fence_before();
    __syncthreads();

    // Instruction descriptors (A operand from shared memory: *_SS; from TMEM: *_TS).
    constexpr uint32_t ID_P = ptx::idesc_bf16(128, 64, 0, 0, 0);    // [Q;K] K^T
    constexpr uint32_t ID_W = ptx::idesc_bf16(128, 128, 1, 0, 0);   // K^T [T''_hi; T''_lo]^T  (A MN-major)
    constexpr uint32_t ID_U = ptx::idesc_bf16(128, 128, 1, 0, 0);   // v^T [T'_hi; T'_lo]^T    (A MN-major)
    constexpr uint32_t ID_WS = ptx::idesc_bf16(128, 128, 0, 1, 1);  // -S^T [W_hi^T | W_lo^T]  (A in TMEM, B MN-major)
    constexpr uint32_t ID_WS_HI = ptx::idesc_bf16(128, 64, 0, 1, 1);  // -S_lo^T W_hi^T
    constexpr uint32_t ID_O = ptx::idesc_bf16(128, 64, 0, 0, 0);    // S^T q^T, v_new^T M^T (A in TMEM)
    constexpr uint32_t ID_S = ptx::idesc_bf16(128, 128, 0, 1, 0);   // v_new'^T K   (A in TMEM, B MN-major)
    // shared-memory descriptors (SW128, SBO 1024) by byte offset from sb, one per LBO
    const uint32_t dlo16 = ptx::sw128_desc_lo(sb, 16), dlo8k = ptx::sw128_desc_lo(sb, 8192),
                   dlo16k = ptx::sw128_desc_lo(sb, 16384);
    auto desc = [](uint32_t lo_base, uint32_t off) { return ptx::desc_pair(lo_base + (off >> 4), ptx::sw128_desc_hi(1024)); };

    for (int n = 0; n < NC; ++n) {
        if (*abort_flag) break;
        const int valid = min(CS, len - n * CS);
        const long long tok0 = tok_base + (long long)n * CS;
        const uint32_t ph = (uint32_t)(n & 1);
        float* rec = (kDebug && p.dbg != nullptr) ? p.dbg + (((size_t)seq * p.HV + h) * p.max_nc + n) * DBG_REC : nullptr;

        // ---- gates: in-chunk inclusive cumsum of g (warp scan), decay factors ----
        if (warp == 1) {  // warp 1: thread 0 (warp 0) issues P1 meanwhile
            float g0, g1, b0, b1;
            gate_of(2 * lane < valid, gn0, bn0, an0, bh0, g0, b0);
            gate_of(2 * lane + 1 < valid, gn1, bn1, an1, bh1, g1, b1);
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

        if constexpr (kPhi) {
            // ---- identity run: no chunk preparation; chunk n's k tile, and its W^T tiles as the
            //      zero-state run of this (segment, head) formed them ----
            wait_bar(BAR_K, ph);
            wait_bar(BAR_V, ph);
            __syncthreads();  // the gates are visible, and every thread is past this chunk's waits
            if (*abort_flag) break;
            if (tid == 0 && n + 1 < NC) load_k(n + 1);  // into the other half of the panels
        } else {
        // ---- P1: [Q;K] K^T (a state pass loads no q: rows 0-63 of the product are not read) ----
        if (!kLean) wait_bar(BAR_Q, ph);
        wait_bar(BAR_K, ph);
        if (kPrestage) {
            // fp16 q/k rows -> fp32 L2 normalisation (eps 1e-6 inside the rsqrt) -> bf16, in
            // place; two threads per row (64 elements each), rows 0-63 q, 64-127 k.
            const int r = tid >> 1, hf = tid & 1;
            float x[64];
            float ss = 0.f;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                uint32_t w4[4];
                ld_shared_v4(sb + OFF_QK + sw_chunk(r, 8 * hf + c, 128), w4[0], w4[1], w4[2], w4[3]);
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const __half2 h2 = *reinterpret_cast<const __half2*>(&w4[u]);
                    x[8 * c + 2 * u] = __low2float(h2);
                    x[8 * c + 2 * u + 1] = __high2float(h2);
                    ss = fmaf(x[8 * c + 2 * u], x[8 * c + 2 * u], ss);
                    ss = fmaf(x[8 * c + 2 * u + 1], x[8 * c + 2 * u + 1], ss);
                }
            }
            ss += __shfl_xor_sync(0xffffffffu, ss, 1);
            const float inv = rsqrtf(ss + 1e-6f);
#pragma unroll
            for (int c = 0; c < 8; ++c)
                st_shared_v4(sb + OFF_QK + sw_chunk(r, 8 * hf + c, 128), pack_bf16(x[8 * c] * inv, x[8 * c + 1] * inv),
                             pack_bf16(x[8 * c + 2] * inv, x[8 * c + 3] * inv),
                             pack_bf16(x[8 * c + 4] * inv, x[8 * c + 5] * inv),
                             pack_bf16(x[8 * c + 6] * inv, x[8 * c + 7] * inv));
            ptx::fence_proxy_async_smem();
            __syncthreads();
        }
        if (tid == 0) {
            ptx::tc_fence_after();
#pragma unroll
            for (int s = 0; s < 8; ++s) {
                const uint32_t koff = (uint32_t)(s >> 2) * 16384u + (uint32_t)(s & 3) * 32u;
                const uint64_t a = desc(dlo16, OFF_QK + koff);
                const uint64_t b = desc(dlo16, OFF_QK + 8192 + koff);
                ptx::mma_bf16(tmem + TM_P, a, b, ID_P, s > 0);
            }
            commit();
        }
        __syncthreads();  // c_s / beta_s visible
        wait_mma();
        {   // rows 0-63: M = scale (q_i.k_j) e^{c_i-c_j}, j <= i (hi/lo); rows 64-127: L
            float v[32];
            ptx::tmem_ld32(tl + TM_P + 32 * half, v);
            ptx::tmem_wait_ld();
            if (row < CS) {
              if (!kLean) {
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
            } else if (!kPrepped) {  // L row i: beta_i k_i.k_j e^{c_i - c_j}, j < i
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
        if (kState && tid == 0 && n > 0) ptx::bulk_wait_read_all();  // the last record's stores have read T', W^T
        ptx::tc_fence_before();
        __syncthreads();
        if constexpr (kPrepped) {
            // ---- this chunk's T' and W^T as the zero-state run formed them; the v^T T'^T part of C12 ----
            wait_bar(BAR_V, ph);
            wait_bar(BAR_W, ph);
            ptx::fence_proxy_async_smem();  // the M tiles, before the async proxy reads them
            __syncthreads();
            if (*abort_flag) break;
            if (tid == 0) {
                ptx::tc_fence_after();
#pragma unroll
                for (int s = 0; s < 4; ++s) {
                    const uint64_t a = desc(dlo8k, OFF_V + s * 2048);
                    const uint64_t b = desc(dlo16, OFF_TP_HI + s * 32);
                    ptx::mma_bf16(tmem + TM_C12, a, b, ID_U, s > 0);
                }
            }
        } else {
        // ---- T = (I + L)^-1 (fp32, CUDA cores) ----
        invert_unit_lower<true>(Ls, X, tid, [](int) {}, [] { __syncthreads(); });
        if (rec) {
            for (int e = tid; e < CS * CS; e += NTHREADS) rec[DBG_T + e] = Ls[(e >> 6) * LSTRIDE + (e & 63)];
            if (tid < CS) rec[DBG_C + tid] = c_s[tid];
        }
        // T' = T diag(beta), T'' = T diag(beta e^c): hi/lo bf16 tiles [64][64]
        {
            const int i = tid >> 2, jb = tid & 3;
            float tp[16], tpp[16];
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {  // two columns per packed multiply
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
                put8_split(sb + OFF_TP_HI + co, sb + OFF_TP_LO + co, tp + 8 * hh, true);
                put8_split(sb + OFF_TPP_HI + co, sb + OFF_TPP_LO + co, tpp + 8 * hh, true);
            }
        }
        if (!phi_unit) wait_bar(BAR_V, ph);
        if (kPrestage) {  // fp16 v -> bf16 in place (gdnChunkPrefillSm87.cu:88-98); each thread its own words
#pragma unroll
            for (int e = tid; e < 1024; e += NTHREADS) {
                uint32_t w4[4];
                const uint32_t a = sb + OFF_V + (uint32_t)e * 16;
                ld_shared_v4(a, w4[0], w4[1], w4[2], w4[3]);
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const __half2 h2 = *reinterpret_cast<const __half2*>(&w4[u]);
                    w4[u] = pack_bf16(__low2float(h2), __high2float(h2));
                }
                st_shared_v4(a, w4[0], w4[1], w4[2], w4[3]);
            }
        }
        ptx::fence_proxy_async_smem();
        __syncthreads();

        // ---- P3: W^T = K^T [T''_hi; T''_lo]^T: cols 0-63 the hi part, 64-127 the lo part ----
        if (tid == 0) {
            ptx::tc_fence_after();
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                const uint64_t a = desc(dlo16k, OFF_QK + 8192 + s * 2048);
                const uint64_t b = desc(dlo16, OFF_TPP_HI + s * 32);  // 128 rows: hi then lo
                ptx::mma_bf16(tmem + TM_W, a, b, ID_W, s > 0);
            }
            commit();
            // C12's state-free part v^T [T'_hi; T'_lo]^T into the dS columns (dS of the previous
            // chunk has been read): cols 0-63 the hi terms, 64-127 the lo terms (B stacked along N).
            // The next commit (after C12's state part) covers it. (Zero in an identity run.)
            if (!phi_unit) {
#pragma unroll
                for (int s = 0; s < 4; ++s) {
                    const uint64_t a = desc(dlo8k, OFF_V + s * 2048);
                    const uint64_t b = desc(dlo16, OFF_TP_HI + s * 32);
                    ptx::mma_bf16(tmem + TM_C12, a, b, ID_U, s > 0);
                }
            }
        }
        wait_mma();
        {   // thread (dk = row, half): W^T[dk][tok] for tok in [32*half, +32), written as rows of W^T
            float v[32], v2[32];
            ptx::tmem_ld32(tl + TM_W + 32 * half, v);
            ptx::tmem_ld32(tl + TM_W + 64 + 32 * half, v2);
            ptx::tmem_wait_ld();
#pragma unroll
            for (int jj = 0; jj < 32; jj += 2)
                    f2_unpack(f2_add(f2_pack(v[jj], v[jj + 1]), f2_pack(v2[jj], v2[jj + 1])), v[jj], v[jj + 1]);
#pragma unroll
            for (int ch = 0; ch < 4; ++ch) {
                const uint32_t co = sw_chunk(row, 4 * half + ch, 128);
                put8_split(sb + OFF_W_HI + co, sb + OFF_W_LO + co, v + 8 * ch, true);
            }
            if (rec) {
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) rec[DBG_W + (32 * half + jj) * HD + row] = v[jj];
            }
        }
        ptx::tc_fence_before();
        ptx::fence_proxy_async_smem();
        __syncthreads();
        if (*abort_flag) break;
        if (kState && tid == 0) {  // this chunk's record, for the identity runs and the output pass
            ptx::bulk_store_s2g(p.wbuf + wrec(n), sb + OFF_TP_HI, 16384);
            ptx::bulk_store_s2g(p.wbuf + wrec(n) + 16384, sb + OFF_W_HI, 32768);
        }
        }  // inverse, T' / T'', P3 and W^T
        }  // chunk preparation

        // ---- C12: v_new^T = v^T T'^T - S^T W^T (the v^T T'^T part was issued with P3) ----
        if (tid == 0) {
            ptx::tc_fence_after();
            // S_hi [W_hi | W_lo], then S_lo W_hi (N = 64: the S_lo W_lo term is below the precision
            // of the split and is left out); S^T from TMEM, W^T tiles MN-major (LBO = 16 KB)
#pragma unroll
            for (int part = 0; part < 2; ++part) {
                const uint32_t sa = part ? TM_SA_LO : TM_SA_HI;
#pragma unroll
                for (int s = 0; s < 8; ++s) {
                    const uint64_t b = desc(dlo16k, (kPhi ? wtile(n) : OFF_W_HI) + s * 2048);
                    // an identity run has no v^T T'^T term: its first product initialises the columns
                    ptx::mma_bf16_ts(tmem + TM_C12, tmem + sa + 8 * s, b, part ? ID_WS_HI : ID_WS,
                                     (!phi_unit || (part | s) > 0) ? 1u : 0u);
                }
            }
            commit();
        }
        // ---- gate = w * silu(z) for this chunk's epilogue, by every thread while C12 runs (the
        //      SFU-bound product slowed the triangular inverse by ~1.6 K cycles when warps 4-7 ran
        //      it alongside; here the warps would otherwise only wait for the MMAs) ----
        if (p.gated) {
            wait_bar(BAR_Z, ph);
            for (int u = tid; u < CS * 16; u += NTHREADS) {
                const int r = u >> 4, zc = u & 15;
                uint32_t w4[4];
                ld_shared_v4(sb + OFF_Z + sw_chunk(r, zc, 64), w4[0], w4[1], w4[2], w4[3]);
                float gv[8];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    float z0, z1;
                    if (kPrestage) {
                        const __half2 z2 = *reinterpret_cast<const __half2*>(&w4[e]);
                        z0 = __low2float(z2), z1 = __high2float(z2);
                    } else {
                        const __nv_bfloat162 z2 = *reinterpret_cast<const __nv_bfloat162*>(&w4[e]);
                        z0 = __low2float(z2), z1 = __high2float(z2);
                    }
                    gv[2 * e] = w_s[8 * zc + 2 * e] * (z0 * rcpf(1.f + ex2f(-z0 * LOG2E)));
                    gv[2 * e + 1] = w_s[8 * zc + 2 * e + 1] * (z1 * rcpf(1.f + ex2f(-z1 * LOG2E)));
                }
                *reinterpret_cast<float4*>(smem + OFF_GATE + gate_chunk(r, 2 * zc)) =
                    make_float4(gv[0], gv[1], gv[2], gv[3]);
                *reinterpret_cast<float4*>(smem + OFF_GATE + gate_chunk(r, 2 * zc + 1)) =
                    make_float4(gv[4], gv[5], gv[6], gv[7]);
            }
        }
        wait_mma();
        if (tid == 0 && n + 1 < NC && n + 1 != p.withhold_v_chunk && !phi_unit && !*abort_flag)
            load_v(n + 1);  // v tile consumed
        if (kPhi && tid == 0 && n + 1 < NC && !*abort_flag) load_w(n + 1);  // C12 of chunk n - 1 read that buffer
        if (kPrepped && tid == 0 && n + 1 < NC && !*abort_flag) load_tw(n + 1);  // T' and W^T are read (C12 done)
        {   // v_new^T (fp32, cols TM_C12) -> hi/lo bf16 pairs of v_new and v_new e^{cL-c} (TMEM A operands)
            float v[32];
            {
                float v2[32];
                ptx::tmem_ld32(tl + TM_C12 + 32 * half, v);
                ptx::tmem_ld32(tl + TM_C12 + 64 + 32 * half, v2);
                ptx::tmem_wait_ld();
#pragma unroll
                for (int jj = 0; jj < 32; jj += 2)
                    f2_unpack(f2_add(f2_pack(v[jj], v[jj + 1]), f2_pack(v2[jj], v2[jj + 1])), v[jj], v[jj + 1]);
            }
            if (rec) {
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) rec[DBG_VN + (32 * half + jj) * HD + row] = v[jj];
            }
            if (!kLean) {   // v_new hi/lo -> cols [0, 64) (the consumed P1 accumulator), for v_new^T M^T
                uint32_t vh[16], vl[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) split2x(v[2 * j], v[2 * j + 1], vh[j], vl[j]);
                ptx::tmem_st16(tl + TM_VN_HI + 16 * half, vh);
                ptx::tmem_st16(tl + TM_VN_LO + 16 * half, vl);
            }
            uint32_t ph_[16], pl[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                float w0, w1;
                f2_unpack(f2_mul(f2_pack(v[2 * j], v[2 * j + 1]), f2_pack(ed_s[32 * half + 2 * j], ed_s[32 * half + 2 * j + 1])), w0, w1);
                split2x(w0, w1, ph_[j], pl[j]);
            }
            ptx::tmem_st16(tl + TM_VP_HI + 16 * half, ph_);
            ptx::tmem_st16(tl + TM_VP_LO + 16 * half, pl);
            ptx::tmem_wait_st();
        }
        ptx::tc_fence_before();
        __syncthreads();
        if (tid == 128 && p.gated && n + 1 < NC && !*abort_flag) {  // every thread is done with the z tile
            ptx::fence_proxy_async_smem();
            load_z(n + 1);
        }
        if (*abort_flag) break;

        // ---- C4: dS^T = v_new'^T K ; C3: o1^T = S^T q^T, o2^T = v_new^T M^T. dS first, each group
        //      with its own commit, so that the state update overlaps the output products ----
        if (tid == 0) {
            ptx::tc_fence_after();
#pragma unroll
            for (int part = 0; part < 2; ++part) {
                const uint32_t va = part ? TM_VP_LO : TM_VP_HI;
#pragma unroll
                for (int s = 0; s < 4; ++s) {
                    const uint64_t b = desc(dlo16k, OFF_QK + koff(n) + s * 2048);
                    ptx::mma_bf16_ts(tmem + TM_S, tmem + va + 8 * s, b, ID_S, (part | s) > 0);
                }
            }
            commit_to(BAR_DS);
            if (!kLean) {
                ptx::mbar_arrive(bar(BAR_DSI));  // dS is in the tensor pipe ahead of the output products
#pragma unroll
                for (int part = 0; part < 2; ++part) {
                    const uint32_t sa = part ? TM_SA_LO : TM_SA_HI;
#pragma unroll
                    for (int s = 0; s < 8; ++s) {
                        const uint64_t b = desc(dlo16, OFF_QK + (s >> 2) * 16384 + (s & 3) * 32);
                        ptx::mma_bf16_ts(tmem + TM_O, tmem + sa + 8 * s, b, ID_O, (part | s) > 0);
                    }
                }
                commit_to(BAR_O1);
            }
        } else if (tid == 32 && !kLean) {
            // v_new^T M^T on a second issuing thread: an MMA issue occupies its thread for about the
            // instruction's execution time, and on thread 0 alone the 36 MMAs held warp 0 back from
            // its state update. (VN_hi, M_hi), (VN_lo, M_hi), (VN_hi, M_lo)
            wait_bar(BAR_DSI, consumed[BAR_DSI] & 1u);
            ptx::tc_fence_after();
            if (!*abort_flag) {  // (after a failed wait nothing more is issued; the consumers' waits run out)
#pragma unroll
            for (int term = 0; term < 3; ++term) {
                const uint32_t va = (term == 1) ? TM_VN_LO : TM_VN_HI;
                const uint32_t mb = (term == 2) ? OFF_M_LO : OFF_M_HI;
#pragma unroll
                for (int s = 0; s < 4; ++s) {
                    const uint64_t b = desc(dlo16, mb + s * 32);
                    ptx::mma_bf16_ts(tmem + TM_O2, tmem + va + 8 * s, b, ID_O, (term | s) > 0);
                }
            }
            commit_to(BAR_O2);
            }
        }
        wait_bar(BAR_DS, consumed[BAR_DS] & 1u);
        ptx::tc_fence_after();

        // ---- state update: S <- e^{cL} S + dS; new S^T hi/lo into TMEM ----
        {
            const float gam = ec_s[CS - 1];
            if (rec) {
#pragma unroll
                for (int j = 0; j < 64; ++j) rec[DBG_SC + (64 * half + j) * HD + row] = S[j];
            }
#pragma unroll
            for (int c2 = 0; c2 < 2; ++c2) {
                float v[32];
                ptx::tmem_ld32(tl + TM_S + 64 * half + 32 * c2, v);
                ptx::tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 32; ++j) S[32 * c2 + j] = fmaf(gam, S[32 * c2 + j], v[j]);
            }
        }
        if (kLean) {  // C12 has read the old state operand and dS the k tile
            if (kState && tid == 0 && n + 1 < NC && !*abort_flag) load_k(n + 1);
            store_state_operand();
            ptx::tmem_wait_st();
            ptx::tc_fence_before();
            __syncthreads();
            continue;
        }
        wait_bar(BAR_O1, consumed[BAR_O1] & 1u);  // S^T q^T has read the old state operand and q
        ptx::tc_fence_after();
        if (tid == 0 && n + 1 < NC && !*abort_flag) {  // q and k tiles consumed (k by dS)
            load_q(n + 1);
            load_k(n + 1);
        }
        store_state_operand();  // new S^T hi/lo for the next chunk's C12 / C3, while v_new^T M^T runs
        wait_bar(BAR_O2, consumed[BAR_O2] & 1u);  // v_new^T M^T done
        ptx::tc_fence_after();

        // ---- o = scale e^c o1 + o2, rounded to bf16, staged [tok][dv] in the (free) L region ----
        {
            float v[32], v2[32];
            ptx::tmem_ld32(tl + TM_O + 32 * half, v);
            ptx::tmem_ld32(tl + TM_O2 + 32 * half, v2);
            ptx::tmem_wait_ld();
            const int dv = row;
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) v[jj] = fmaf(p.scale * ec_s[32 * half + jj], v[jj], v2[jj]);
            if (rec) {
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) rec[DBG_O + (32 * half + jj) * HD + dv] = v[jj];
            }
            __nv_bfloat16* ot = reinterpret_cast<__nv_bfloat16*>(smem + OFF_OST);
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) ot[sw_off(32 * half + jj, dv, 64) >> 1] = __float2bfloat16_rn(v[jj]);
        }
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        __syncthreads();

        // ---- epilogue: 4 threads per token, 16-byte chunks {eq, eq+4, eq+8, eq+12} ----
        {
            float o[32];
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                uint32_t w4[4];
                ld_shared_v4(sb + OFF_OST + sw_chunk(et, eq + 4 * m, 64), w4[0], w4[1], w4[2], w4[3]);
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const __nv_bfloat162 b2 = *reinterpret_cast<const __nv_bfloat162*>(&w4[u]);
                    o[8 * m + 2 * u] = __bfloat162float(b2.x);
                    o[8 * m + 2 * u + 1] = __bfloat162float(b2.y);
                }
            }
            uint32_t outw[16];
            // Output rounding: bf16, or in pre-stage mode fp16 (o is already a bf16 value,
            // exactly representable in fp16 inside its range, as the adapter's bf16->fp16 bridge).
            auto pack_out = [&](float a, float b) -> uint32_t {
                if (kPrestage) {
                    const __half2 h2 = __floats2half2_rn(a, b);
                    return *reinterpret_cast<const uint32_t*>(&h2);
                }
                return pack_bf16(a, b);
            };
            auto round_in = [&](float x) -> float {  // the norm's round-to-input-dtype step
                return kPrestage ? __half2float(__float2half_rn(x)) : bf16r(x);
            };
            if (!p.gated) {
#pragma unroll
                for (int j = 0; j < 16; ++j) outw[j] = pack_out(o[2 * j], o[2 * j + 1]);
            } else {
                if (kPrestage) {  // the norm reads the adapter's fp16 o (bf16 -> fp16 bridge, subnormals included)
#pragma unroll
                    for (int j = 0; j < 32; ++j) o[j] = __half2float(__float2half_rn(o[j]));
                }
                float ss = 0.f;
#pragma unroll
                for (int j = 0; j < 32; ++j) ss = fmaf(o[j], o[j], ss);
                ss += __shfl_xor_sync(0xffffffffu, ss, 1);
                ss += __shfl_xor_sync(0xffffffffu, ss, 2);
                const float rstd = rsqrtf(ss * (1.f / (float)HD) + p.eps);
#pragma unroll
                for (int m = 0; m < 4; ++m) {
                    const int c = eq + 4 * m;
                    const float4 g0 = *reinterpret_cast<const float4*>(smem + OFF_GATE + gate_chunk(et, 2 * c));
                    const float4 g1 = *reinterpret_cast<const float4*>(smem + OFF_GATE + gate_chunk(et, 2 * c + 1));
                    const float gg[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        outw[4 * m + e] = pack_out(round_in(o[8 * m + 2 * e] * rstd) * gg[2 * e],
                                                   round_in(o[8 * m + 2 * e + 1] * rstd) * gg[2 * e + 1]);
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
    }

    // ---- final state: at (seq, h); in a state pass at (segment, grid row) of its 2 HV rows; in an
    //      output pass only the last segment's, at (batch row, h) ----
    if (!*abort_flag) {
        float* sfp = p.sf + ((size_t)seq * p.HV + h) * HD * HD;
        if (kLean)  // the [b (seg_total - 1) + j][2 HV] maps; the last segment's zero-state run has none
            sfp = seg_j < p.seg_total - 1
                      ? p.sf + (((size_t)bcoord * (p.seg_total - 1) + seg_j) * 2 * p.HV + (kPhi ? p.HV : 0) + h) * HD * HD
                      : nullptr;
        if (kSeg == SEG_OUTPUT)
            sfp = (seq % p.seg_per_seq == p.seg_per_seq - 1) ? p.sf + ((size_t)(seq / p.seg_per_seq) * p.HV + h) * HD * HD
                                                            : nullptr;
        if (phi_unit && sfp != nullptr) {  // the map Phi is stored transposed, PhiT[k][i] = Phi[i][k] (k = row): the scan's layout
            float4* dst = reinterpret_cast<float4*>(sfp + (size_t)row * HD + 64 * half);
#pragma unroll
            for (int j = 0; j < 16; ++j) dst[j] = make_float4(S[4 * j], S[4 * j + 1], S[4 * j + 2], S[4 * j + 3]);
        } else if (sfp != nullptr) {
#pragma unroll
            for (int j = 0; j < 64; ++j) {
                const int dk = 64 * half + j;
                sfp[(size_t)dk * HD + row] = S[j];
            }
        }
    }
    if (kState && tid == 0) ptx::bulk_wait_all();  // the records' stores have completed
    // Abort path: wait (bounded) for this CTA's own TMA copies and MMAs still
    // in flight before its shared memory and TMEM are released.
    if (*abort_flag && (tid == 0 || tid == 32 || tid == 128)) {
#pragma unroll
        for (int i = 0; i < NBAR; ++i)
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
static bool make_map(CUtensorMap* m, const void* base, int H, int T, int B, bool fp16 = false) {
    EncodeTiledFn enc = get_encode_fn();
    if (!enc) return false;
    cuuint64_t dims[4] = {(cuuint64_t)HD, (cuuint64_t)H, (cuuint64_t)T, (cuuint64_t)B};
    cuuint64_t strides[3] = {(cuuint64_t)HD * 2, (cuuint64_t)H * HD * 2, (cuuint64_t)T * H * HD * 2};
    cuuint32_t box[4] = {64, 1, 64, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = enc(m, fp16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4,
                     const_cast<void*>(base), dims, strides,
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
    for (auto fn : {gdn_prefill_kernel<false, false>, gdn_prefill_kernel<true, false>, gdn_prefill_kernel<false, true>,
                    gdn_prefill_kernel<true, true>, gdn_prefill_kernel<false, false, SEG_OUTPUT>,
                    gdn_prefill_kernel<false, false, SEG_STATE>, gdn_prefill_kernel<false, false, SEG_PHI>}) {
        e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_ALLOC);
        if (e != cudaSuccess) break;
    }
    if (e == cudaSuccess && bit) done_mask.fetch_or(bit, std::memory_order_acq_rel);
    return e;
}

constexpr size_t WS_HEADER = 256;

cudaError_t launch_split(const Params& p, int nseq, int grid_heads, cudaStream_t stream);  // gdn_prefill_split.cu
cudaError_t launch_segment_scan(const float* stt, const float* s0, float* entry, int B, int HV, int nseg,
                                cudaStream_t stream);  // gdn_segment_scan.cu
int split_cluster_ctas();
int split_clusters_per_wave();
bool split_available();

// Kernel choice: the cluster-split kernel when the (sequence, head) clusters run
// in at most two waves, else the one-CTA-per-head kernel. Small batches are
// latency-bound on the state chain: measured on B200, a cluster takes ~3.5 us per
// chunk and the one-CTA kernel ~11.5 us, so two waves of clusters (B=2, HV=32:
// 181 vs 233 us at S=1141) still win, three are about even, and with more
// (sequence, head) units than SMs the one-CTA kernel uses the GPU better.
// GDN_B200_KERNEL=fused|split|auto overrides (debug dumps and the pre-stage mode
// use the one-CTA kernel). A forced split launch fails with cudaErrorNotSupported
// when the compiled split kernel does not have the register count its register
// split is written for.
static bool use_split(int nseq, int HV, int force) {
    if (force == 1) return false;
    if (force == 2) return split_available();
    const char* env = getenv("GDN_B200_KERNEL");
    if (env && strcmp(env, "fused") == 0) return false;
    if (env && strcmp(env, "split") == 0) return true;
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return false;
    const long long per_wave = sms / split_cluster_ctas();
    return per_wave > 0 && (long long)nseq * HV <= 2 * per_wave && split_available();
}

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
    // pre-stage (adapter) inputs
    int prestage;
    const void *ga, *gb, *dt_bias;
    const float* A_log;
    // test hook (deltanet_test_withheld_load): kernel choice (0 automatic, 1 one CTA per head,
    // 2 cluster split) and the chunk whose v-tile load is withheld (-1 none)
    int force_kernel;
    int withhold_v_chunk;
    // segmented passes (deltanet_chunk_prefill_segmented): chunks per segment and segments per
    // sequence (nseq = B * seg_per_seq); the state pass (2 HV heads in the grid, no output; the
    // cluster-split kernel reads the identity runs' v through the zero tile v0) or the output pass
    // (only the last segment's final state, at sf[b]); seg_kernel 1: one CTA per unit, 2: cluster split
    int seg_chunks, seg_per_seq;
    int state_pass;
    const void* v0;
    int sf_last_only;
    int seg_kernel;
    // one-CTA segmented state passes: the zero-state runs (state_pass) store W^T tiles to wbuf, the
    // identity runs' pass (phi_pass) reads them
    int phi_pass;
    void* wbuf;
    int seg_total;  // segments per sequence of the whole call (record and map indexing)
};

// A Launch with every field cleared and no test hook armed.
static Launch blank_launch() {
    Launch L;
    memset(&L, 0, sizeof(L));
    L.withhold_v_chunk = -1;
    return L;
}

static cudaError_t launch(const Launch& L) {
    if (L.DK != HD || L.DV != HD || L.chunk != CS) return cudaErrorInvalidValue;
    if (L.HQK <= 0 || L.HV <= 0 || L.HV % L.HQK != 0) return cudaErrorInvalidValue;
    if (L.T < 0 || L.nseq < 0 || L.HV > 65535 || L.nseq > 65535) return cudaErrorInvalidValue;
    if (!L.q || !L.k || !L.v || (!L.out && !L.state_pass && !L.phi_pass) || !L.sf || !L.ws) return cudaErrorInvalidValue;
    if (L.state_pass && ((L.seg_kernel == 2 && !L.v0) || L.seg_chunks <= 0 || L.s0)) return cudaErrorInvalidValue;
    if (L.seg_chunks > 0 && L.seg_kernel == 1 && (!L.wbuf || !aligned16(L.wbuf) || L.seg_total < 2)) return cudaErrorInvalidValue;
    if (L.phi_pass && (L.seg_kernel != 1 || L.state_pass || L.s0 || L.seg_chunks <= 0)) return cudaErrorInvalidValue;
    if (L.prestage ? (!L.ga || !L.gb || !L.A_log || !L.dt_bias) : (!L.g || !L.beta)) return cudaErrorInvalidValue;
    if (L.ws_bytes < WS_HEADER) return cudaErrorInvalidValue;
    const bool gated = (L.z != nullptr) || (L.w != nullptr);
    if (gated && (!L.z || !L.w)) return cudaErrorInvalidValue;
    if (!aligned16(L.q) || !aligned16(L.k) || !aligned16(L.v) || (gated && !aligned16(L.z)) ||
        !aligned16(L.ws) || !aligned16(L.out) || !aligned16(L.v0))
        return cudaErrorInvalidValue;
    if (L.nseq == 0 || L.HV == 0) return cudaSuccess;

    Params p;
    memset(&p, 0, sizeof(p));
    const int Bmap = L.cu ? 1 : L.B;
    const int Tmap = L.T > 0 ? L.T : 1;
    const bool f16 = L.prestage != 0;
    if (!make_map(&p.tm_q, L.q, L.HQK, Tmap, Bmap, f16) || !make_map(&p.tm_k, L.k, L.HQK, Tmap, Bmap, f16) ||
        !make_map(&p.tm_v, L.v, L.HV, Tmap, Bmap, f16))
        return cudaErrorInvalidValue;
    if (gated) {
        if (!make_map(&p.tm_z, L.z, L.HV, Tmap, Bmap, f16)) return cudaErrorInvalidValue;
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
    p.prestage = L.prestage;
    p.ga = static_cast<const __half*>(L.ga);
    p.gb = static_cast<const __half*>(L.gb);
    p.A_log = L.A_log;
    p.dt_bias = static_cast<const __half*>(L.dt_bias);
    p.withhold_v_chunk = L.withhold_v_chunk;
    p.seg_chunks = L.seg_chunks;
    p.seg_per_seq = L.seg_per_seq;
    p.sf_last_only = L.sf_last_only;
    p.wbuf = static_cast<uint8_t*>(L.wbuf);
    p.seg_total = L.seg_total;
    p.tm_v0 = p.tm_v;
    if (L.seg_chunks > 0) {  // segmented passes (the caller checked that the chosen kernel can run)
        if (L.dbg || L.prestage || L.cu || L.nseq != L.B * L.seg_per_seq) return cudaErrorInvalidValue;
        if ((L.state_pass || L.phi_pass) && gated) return cudaErrorInvalidValue;
        if (L.seg_kernel == 2) {
            if (L.state_pass && !make_map(&p.tm_v0, L.v0, 1, CS, 1)) return cudaErrorInvalidValue;  // one zero tile
            return launch_split(p, L.nseq, L.state_pass ? 2 * L.HV : L.HV, L.stream);
        }
        if (L.seg_kernel != 1) return cudaErrorInvalidValue;
    }

    const bool split = L.seg_chunks == 0 && !L.dbg && !L.prestage && use_split(L.nseq, L.HV, L.force_kernel);
    if (L.force_kernel == 2 && !split) return cudaErrorNotSupported;
    if (split) return launch_split(p, L.nseq, L.HV, L.stream);
    cudaError_t e = ensure_smem_attr();
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(1, L.HV, L.nseq);
    cfg.blockDim = dim3(NTHREADS, 1, 1);
    cfg.dynamicSmemBytes = SMEM_ALLOC;
    cfg.stream = L.stream;
    // programmatic dependent launch: the kernel waits for the previous grid before touching memory
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void (*kernel)(Params) = L.prestage ? (L.dbg ? gdn_prefill_kernel<true, true> : gdn_prefill_kernel<true, false>)
                                        : (L.dbg ? gdn_prefill_kernel<false, true> : gdn_prefill_kernel<false, false>);
    if (L.seg_chunks > 0)
        kernel = L.state_pass ? gdn_prefill_kernel<false, false, SEG_STATE>
                              : (L.phi_pass ? gdn_prefill_kernel<false, false, SEG_PHI>
                                            : gdn_prefill_kernel<false, false, SEG_OUTPUT>);
    e = cudaLaunchKernelEx(&cfg, kernel, p);
    if (e != cudaSuccess) return e;
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
static_assert(WS_HEADER <= NOALLOC_SCRATCH_BYTES, "the static scratch must hold the status header");

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

// ---------------------------------------------------------------------------
// Long sequences in segments (deltanet_chunk_prefill_segmented).
constexpr size_t SEG_ZERO_BYTES = (size_t)CS * HD * 2;  // one zero bf16 tile [64 tok][128]: the identity runs' v

// Plan of a segmented call: segments per sequence, chunks per segment and the kernel that runs
// the passes (1: one CTA per (segment, head), 2: cluster split), from a wave model of B200
// measurements. A wave of units costs its chunk count plus a start-up and drain overhead, times
// the kernel's chunk period; the call costs the state pass (the zero-state and the identity runs
// of every segment but the last, U (s - 1) units each), the scan (one step per segment) and the
// output pass (U s units), U = B HV.
//   cluster split: 4 SMs per unit, clusters per wave from the occupancy API (32 on B200: clusters
//     must fit inside a GPC), ~3.0 us per chunk in either pass (both runs in one grid), ~5 periods
//     of overhead;
//   one CTA per unit: one unit per SM; the zero-state runs of every segment (~7.4 us per chunk:
//     no output products, norm or q loads), the identity runs (~3.2 us: no chunk preparation, they
//     read the zero-state runs' W) and the output pass (~7.3 us: it reads their T' and W), ~1
//     period of overhead; one pass of the one-CTA kernel costs ~10.2 us per chunk;
//   the scan ~1.7 us per step.
// One pass (s = 1) costs what the plain call launches. The cheapest plan wins, fewer segments on
// ties. GDN_B200_KERNEL=fused|split restricts the passes to one kernel.
struct SegPlan {
    int nseg, per, kernel;
};
constexpr double SPLIT_CHUNK_US = 3.0, FUSED_CHUNK_US = 10.2, STATE_CHUNK_US = 7.4, PHI_CHUNK_US = 3.2,
                 OUTPUT_CHUNK_US = 7.3, SCAN_STEP_US = 1.7;
constexpr int WAVE_OVERHEAD = 5, FUSED_OVERHEAD = 1;
static SegPlan plan_segments(int B, int HV, int NC, int segments, int sms, int cluster_wave, bool split_ok,
                             bool fused_ok) {
    const long long U = (long long)B * HV;
    auto waves = [](long long units, int wave) { return (double)((units + wave - 1) / wave); };
    if (cluster_wave <= 0 || sms <= 0) split_ok = false;
    if (!split_ok) fused_ok = true;  // the one-CTA kernel always runs
    auto cost = [&](int eff, int per, int kernel) {  // segmented call, `eff` segments of `per` chunks
        const double scan = eff * SCAN_STEP_US;
        const long long su = U * (eff - 1);  // units of either run kind: every segment but the last
        if (kernel == 2)
            return (waves(2 * su, cluster_wave) + waves(U * eff, cluster_wave)) * (per + WAVE_OVERHEAD) *
                       SPLIT_CHUNK_US + scan;
        return (waves(U * eff, sms) * (STATE_CHUNK_US + OUTPUT_CHUNK_US) + waves(su, sms) * PHI_CHUNK_US) *
                   (per + FUSED_OVERHEAD) + scan;
    };
    auto cheaper_kernel = [&](int eff, int per) {
        if (!split_ok) return 1;
        if (!fused_ok) return 2;
        return cost(eff, per, 1) <= cost(eff, per, 2) ? 1 : 2;
    };
    SegPlan best{1, NC, 0};
    if (NC <= 1) return best;
    if (segments > 0) {  // an explicit request: that many segments (at most one per chunk), whatever one pass costs
        const int s = segments < NC ? segments : NC;
        const int per = (NC + s - 1) / s, eff = (NC + per - 1) / per;
        if (eff <= 1) return best;
        return SegPlan{eff, per, sms > 0 ? cheaper_kernel(eff, per) : (split_ok ? 2 : 1)};
    }
    if (sms <= 0) return best;
    // one pass: the plain call's kernel choice (cluster split while the clusters fit in two waves)
    double best_cost = (split_ok && U <= 2LL * (sms / 4))
                           ? waves(U, cluster_wave) * (NC + WAVE_OVERHEAD) * SPLIT_CHUNK_US
                           : waves(U, sms) * (NC + FUSED_OVERHEAD) * FUSED_CHUNK_US;
    for (int s = 2; s <= NC && s <= 256; ++s) {
        const int per = (NC + s - 1) / s;
        if ((NC + per - 1) / per != s) continue;  // `per` chunks each make fewer segments
        const int k = cheaper_kernel(s, per);
        const double c = cost(s, per, k);
        if (c < best_cost) {
            best_cost = c;
            best = SegPlan{s, per, k};
        }
    }
    return best;
}

// The plan for a request of `segments` (0: automatic) on the current device.
static SegPlan resolve_segments(int B, int T, int HV, int segments) {
    const int NC = (T + CS - 1) / CS;
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        sms = 0;
    const char* env = getenv("GDN_B200_KERNEL");
    bool split_ok = split_available(), fused_ok = true;
    if (env && strcmp(env, "fused") == 0) split_ok = false;
    if (env && strcmp(env, "split") == 0) fused_ok = false;
    int wave = split_ok ? split_clusters_per_wave() : 0;
    if (split_ok && wave <= 0) wave = sms / split_cluster_ctas();  // no occupancy answer: SMs / cluster size
    SegPlan pl = plan_segments(B, HV, NC, segments, sms, wave, split_ok, fused_ok);
    if (pl.kernel == 0 || pl.nseg <= 1) pl = SegPlan{1, NC, 0};
    return pl;
}

// status header, the zero tile, the state pass's maps A_j and PhiT_j of every segment but the
// last ([B (nseg - 1)][2 HV][128][128] fp32), the entry states ([B nseg][HV][128][128] fp32) and,
// for passes on the one-CTA kernel, the records (T' and W^T tiles) of every chunk of every
// segment ([B nseg][HV][per] x 48 KB)
static size_t seg_maps_bytes(int B, int HV, int nseg) {
    return (size_t)B * (3 * nseg - 2) * HV * HD * HD * sizeof(float);
}
static size_t segmented_bytes(const SegPlan& pl, int B, int HV) {
    if (pl.nseg <= 1) return WS_HEADER;
    const size_t w = pl.kernel == 1 ? (size_t)B * pl.nseg * HV * pl.per * WREC_BYTES : 0;
    return WS_HEADER + SEG_ZERO_BYTES + seg_maps_bytes(B, HV, pl.nseg) + w;
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

size_t deltanet_segmented_workspace_size(int B, int T, int HV, int DK, int DV, int chunk_size, int segments) {
    (void)DK; (void)DV; (void)chunk_size;
    if (B <= 0 || T <= 0 || HV <= 0) return gdn::WS_HEADER;
    return gdn::segmented_bytes(gdn::resolve_segments(B, T, HV, segments), B, HV);
}

// The plan deltanet_chunk_prefill_segmented makes for these sizes on the current device: segments
// per sequence, chunks per segment and the kernel of its passes (0: one pass, the plain call;
// 1: one CTA per (segment, head); 2: cluster split).
cudaError_t deltanet_segmented_plan(int B, int T, int HV, int segments, int* nseg, int* chunks_per_segment,
                                    int* kernel) {
    if (!nseg || !chunks_per_segment || !kernel || segments < 0 || B < 0 || T < 0 || HV <= 0)
        return cudaErrorInvalidValue;
    gdn::SegPlan pl{1, (T + gdn::CS - 1) / gdn::CS, 0};
    if (B > 0 && T > 0) pl = gdn::resolve_segments(B, T, HV, segments);
    *nseg = pl.nseg;
    *chunks_per_segment = pl.per;
    *kernel = pl.kernel;
    return cudaSuccess;
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
    gdn::Launch L = gdn::blank_launch();
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
    gdn::Launch L = gdn::blank_launch();
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
    gdn::Launch L = gdn::blank_launch();
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

// Test hook for the bounded waits: the gated prefill with one v-tile load never issued, so that
// the wait for it runs out (the form of failure the kernels must survive: a producer that never
// arrives). No fault, trap or unbounded wait is involved.
cudaError_t deltanet_test_withheld_load(const void* q, const void* k, const void* v, const float* g,
                                        const float* beta, const void* z, const void* norm_w, float eps,
                                        void* y, const float* initial_state, float* final_state, int B, int T,
                                        int HV, int HQK, int DK, int DV, int chunk_size, void* workspace,
                                        size_t workspace_bytes, cudaStream_t stream, int kernel,
                                        int withheld_chunk) {
    if (!z || !norm_w || kernel < 0 || kernel > 2 || withheld_chunk < 0) return cudaErrorInvalidValue;
    gdn::Launch L = gdn::blank_launch();
    L.q = q; L.k = k; L.v = v; L.g = g; L.beta = beta; L.z = z; L.w = norm_w; L.eps = eps; L.out = y;
    L.s0 = initial_state; L.sf = final_state;
    L.nseq = B; L.B = B; L.T = T; L.HV = HV; L.HQK = HQK; L.DK = DK; L.DV = DV; L.chunk = chunk_size;
    L.max_nc = (T + gdn::CS - 1) / gdn::CS;
    L.ws = workspace; L.ws_bytes = workspace_bytes; L.stream = stream;
    L.force_kernel = kernel;
    L.withhold_v_chunk = withheld_chunk;
    return gdn::launch(L);
}

// Long sequences cut into segments that run side by side (few sequences and heads leave most of
// the GPU idle on the serial chunk recurrence). Three launches on `stream`: the state pass (every
// segment from a zero state, giving A_j, and from the identity with zero v, giving Phi_j, in one
// grid), the scan S_{j+1} = Phi_j S_j + A_j of entry states, and the output pass (every segment
// from its entry state; only the last segment of each sequence writes its final state).
cudaError_t deltanet_chunk_prefill_segmented(const void* q, const void* k, const void* v, const float* g,
                                             const float* beta, const void* z, const void* norm_w, float eps,
                                             void* out, const float* initial_state, float* final_state, int B,
                                             int T, int HV, int HQK, int DK, int DV, int chunk_size, int segments,
                                             void* workspace, size_t workspace_bytes, cudaStream_t stream) {
    if ((z == nullptr) != (norm_w == nullptr) || segments < 0) return cudaErrorInvalidValue;
    if (DK != gdn::HD || DV != gdn::HD || chunk_size != gdn::CS || B < 0 || T < 0 || HV <= 0) return cudaErrorInvalidValue;
    gdn::SegPlan plan{1, 1, 0};
    if (B > 0 && T > 0) plan = gdn::resolve_segments(B, T, HV, segments);
    const int nseg = plan.nseg, per = plan.per;
    if (nseg <= 1)  // one pass is the plain call
        return z ? deltanet_chunk_prefill_gated(q, k, v, g, beta, z, norm_w, eps, out, initial_state, final_state, B, T,
                                                HV, HQK, DK, DV, chunk_size, workspace, workspace_bytes, stream)
                 : deltanet_chunk_prefill(q, k, v, g, beta, out, initial_state, final_state, B, T, HV, HQK, DK, DV,
                                          chunk_size, workspace, workspace_bytes, stream, 0);
    if (!workspace || workspace_bytes < gdn::segmented_bytes(plan, B, HV)) return cudaErrorInvalidValue;
    char* ws = static_cast<char*>(workspace);
    void* zero = ws + gdn::WS_HEADER;
    float* stt = reinterpret_cast<float*>(ws + gdn::WS_HEADER + gdn::SEG_ZERO_BYTES);  // [B (nseg-1)][2 HV][D][D]
    float* entry = stt + (size_t)B * (nseg - 1) * 2 * HV * gdn::HD * gdn::HD;           // [B nseg][HV][D][D]
    cudaError_t e = cudaMemsetAsync(zero, 0, gdn::SEG_ZERO_BYTES, stream);
    if (e != cudaSuccess) return e;
    gdn::Launch L = gdn::blank_launch();
    L.q = q; L.k = k; L.v = v; L.g = g; L.beta = beta; L.eps = eps;
    L.B = B; L.T = T; L.HV = HV; L.HQK = HQK; L.DK = DK; L.DV = DV; L.chunk = chunk_size;
    L.max_nc = per;
    L.ws = workspace; L.ws_bytes = workspace_bytes; L.stream = stream;
    L.seg_chunks = per; L.seg_kernel = plan.kernel; L.seg_total = nseg;
    // State pass: the maps A_j (zero entry, v) at heads [0, HV) and PhiT_j (identity entry, zero v)
    // at [HV, 2 HV) of the segments but the last (whose maps are not needed). The cluster-split
    // kernel runs both in one grid over those segments. The one-CTA kernel runs the zero-state runs
    // of every segment, which store every chunk's record (T' and W^T), then the identity runs,
    // which read W^T from them; the output pass reads T' and W^T from them too.
    L.state_pass = 1; L.v0 = zero; L.sf = stt; L.out = nullptr;
    if (plan.kernel == 1) {
        L.wbuf = ws + gdn::WS_HEADER + gdn::SEG_ZERO_BYTES + gdn::seg_maps_bytes(B, HV, nseg);
        L.nseq = B * nseg; L.seg_per_seq = nseg;
        e = gdn::launch(L);
        if (e != cudaSuccess) return e;
        L.state_pass = 0; L.phi_pass = 1; L.v0 = nullptr;
        L.nseq = B * (nseg - 1); L.seg_per_seq = nseg - 1;
        e = gdn::launch(L);
        if (e != cudaSuccess) return e;
        L.phi_pass = 0;
    } else {
        L.nseq = B * (nseg - 1); L.seg_per_seq = nseg - 1;
        e = gdn::launch(L);
        if (e != cudaSuccess) return e;
    }
    e = gdn::launch_segment_scan(stt, initial_state, entry, B, HV, nseg, stream);
    if (e != cudaSuccess) return e;
    // output pass over every segment from its entry state; the last segment's final state is the sequence's
    L.nseq = B * nseg; L.seg_per_seq = nseg;
    L.state_pass = 0; L.v0 = nullptr; L.z = z; L.w = norm_w; L.out = out;
    L.s0 = entry; L.sf = final_state; L.sf_last_only = 1;
    return gdn::launch(L);
}

int gdn_run_chunk_prefill(const gdn_prefill_params* params, cudaStream_t stream) {
    if (params == nullptr) {
        fprintf(stderr, "gdn_run_chunk_prefill: null params\n");
        return -1;
    }
    const gdn_prefill_params& P = *params;
    if (P.k_dim != gdn::HD || P.v_dim != gdn::HD) {
        fprintf(stderr, "gdn_run_chunk_prefill: requires k_dim=v_dim=128, got %d/%d\n", P.k_dim, P.v_dim);
        return -1;
    }
    if (P.h <= 0 || P.hv <= 0 || P.hv < P.h || P.hv % P.h != 0) {
        fprintf(stderr, "gdn_run_chunk_prefill: requires hv >= h and hv %% h == 0, got h=%d hv=%d\n", P.h, P.hv);
        return -1;
    }
    if (!P.q || !P.k || !P.v || !P.a || !P.b || !P.A_log || !P.dt_bias || !P.h0_source || !P.o) {
        fprintf(stderr, "gdn_run_chunk_prefill: null tensor pointer\n");
        return -1;
    }
    if (P.n <= 0 || P.seq_len <= 0) {
        fprintf(stderr, "gdn_run_chunk_prefill: n and seq_len must be positive, got n=%d seq_len=%d\n", P.n,
                P.seq_len);
        return -1;
    }
    if ((P.z == nullptr) != (P.norm_w == nullptr)) {
        fprintf(stderr, "gdn_run_chunk_prefill: pass both z and norm_w to fuse the norm, or neither\n");
        return -1;
    }
    gdn::Launch L = gdn::blank_launch();
    L.q = P.q; L.k = P.k; L.v = P.v; L.z = P.z; L.w = P.norm_w; L.eps = P.eps; L.out = P.o;
    L.s0 = P.h0_source; L.sf = P.h0_source;  // initial state in, final state out, in place
    L.nseq = P.n; L.B = P.n; L.T = P.seq_len; L.HV = P.hv; L.HQK = P.h; L.DK = P.k_dim; L.DV = P.v_dim;
    L.chunk = gdn::CS; L.max_nc = (P.seq_len + gdn::CS - 1) / gdn::CS;
    L.ws = P.workspace; L.ws_bytes = P.workspace_bytes; L.stream = stream;
    L.prestage = 1; L.ga = P.a; L.gb = P.b; L.A_log = P.A_log; L.dt_bias = P.dt_bias;
    const cudaError_t e = gdn::launch(L);
    if (e != cudaSuccess) {
        fprintf(stderr, "gdn_run_chunk_prefill: %s\n", cudaGetErrorString(e));
        return -1;
    }
    return 0;
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

// Status word of the no-allocation entry's static scratch on the current device: the same
// word deltanet_read_status reads from a caller's workspace (0 = clean, bit 0 = a bounded wait
// timed out), read after the work already queued on `stream` and cleared when clear != 0.
// Reads only the static array: no allocation here either.
cudaError_t deltanet_noalloc_read_status(int* status_host, int clear, cudaStream_t stream) {
    if (!status_host) return cudaErrorInvalidValue;
    void* ws = nullptr;
    cudaError_t e = gdn::noalloc_scratch(&ws);
    if (e != cudaSuccess) return e;
    return deltanet_read_status(ws, status_host, clear, stream);
}

const char* gdn_b200_version(void) { return "gdn_b200 0.1 (sm_100a, tcgen05 fused prefill)"; }

}  // extern "C"
