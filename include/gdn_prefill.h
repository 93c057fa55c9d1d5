/*
 * gdn_b200 C ABI: chunked gated-delta-rule (gated DeltaNet) prefill with a fused
 * gated-RMSNorm epilogue, for NVIDIA B200 (sm_100a).
 *
 * Drop-in for the reference's kernel C ABI (kernels/chunk_delta_cuda.h:39-55 and
 * its twin kernels/chunk_delta_cuda_tco.h:39-55): same names, argument order,
 * types and error convention. All buffers are caller-owned, contiguous device
 * memory; calls are asynchronous and stream-ordered; nothing is allocated.
 *
 * IO contract (unchanged from kernels/chunk_delta_cuda.h:11-27):
 *   q, k : bf16 [B, T, HQK, DK]   pre-L2-normalised; v-head h reads qk-head h / (HV/HQK)
 *   v    : bf16 [B, T, HV, DV]
 *   g    : fp32 [B, T, HV]        log-decay (<= 0), cumsummed inside 64-token chunks
 *   beta : fp32 [B, T, HV]
 *   o    : bf16 [B, T, HV, DV]    out
 *   s0   : fp32 [B, HV, DK, DV] or NULL (zeros);   sf : fp32 [B, HV, DK, DV] out
 * The kernel applies the 1/sqrt(DK) query scale itself
 * (kernels/chunk_delta_cuda.cu:805,811). Only DK = DV = 128 and chunk_size = 64
 * are supported; anything else returns cudaErrorInvalidValue.
 *
 * Errors: cudaErrorInvalidValue for unsupported dimensions, HV % HQK != 0, NULL
 * required pointers, a NULL or short workspace, or misaligned pointers
 * (tensors must be 16-byte aligned); otherwise the launch error, if any.
 * A device-side status word in the workspace records bounded-wait timeouts
 * (read it with deltanet_read_status).
 */
#ifndef GDN_B200_GDN_PREFILL_H_
#define GDN_B200_GDN_PREFILL_H_

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Workspace bytes for one prefill call (status header). Replaces
 * deltanet_prefill_workspace_size, kernels/chunk_delta_cuda.h:40. The fused
 * kernel keeps every chunk intermediate on chip, so the size no longer scales
 * with B*HV*NC (the reference needs ~123 MB at B=1, T=1141, HV=32). */
size_t deltanet_prefill_workspace_size(int B, int T, int HV, int DK, int DV, int chunk_size);

/* Workspace bytes when dump_debug != 0: the header plus one fp32 record per
 * (b, h, chunk) = [c(64) | T(64x64) | W(64x128) | v_new(64x128) | o(64x128) |
 * S_entry(128x128)]. No counterpart in the reference (its debug dumps are
 * always carried in the workspace, kernels/chunk_delta_cuda.cu:688-697, in its
 * own carve-out of w | u | de | eg | ed | gl | Sc | M | T | A | T-post-leaf).
 * The torch binding's chunk_prefill_debug forms the reference's views from
 * this record (u = W, Sc = S_entry, T, and de / eg / ed / gl from c) and the
 * inputs (w, M, A, T-post-leaf), in the reference's order and shapes. */
size_t deltanet_prefill_debug_workspace_size(int B, int T, int HV, int DK, int DV, int chunk_size);

/* Chunked gated delta rule prefill, o written in bf16. Replaces
 * deltanet_chunk_prefill, kernels/chunk_delta_cuda.h:46-55 (identical signature). */
cudaError_t deltanet_chunk_prefill(
    const void* q, const void* k, const void* v,
    const float* g, const float* beta,
    void* o,
    const float* initial_state,
    float* final_state,
    int B, int T, int HV, int HQK, int DK, int DV, int chunk_size,
    void* workspace, size_t workspace_bytes,
    cudaStream_t stream, int dump_debug);

/* The reference's production ("TCO", bf16 o-pass) entry points,
 * kernels/chunk_delta_cuda_tco.h:40-55. Same math and contract; aliases of the
 * two functions above. */
size_t deltanet_tcop_prefill_workspace_size(int B, int T, int HV, int DK, int DV, int chunk_size);
cudaError_t deltanet_tcop_chunk_prefill(
    const void* q, const void* k, const void* v,
    const float* g, const float* beta,
    void* o,
    const float* initial_state,
    float* final_state,
    int B, int T, int HV, int HQK, int DK, int DV, int chunk_size,
    void* workspace, size_t workspace_bytes,
    cudaStream_t stream, int dump_debug);

/* Prefill with the gated RMSNorm fused as the epilogue: o never reaches HBM.
 *   y = bf16( w * bf16(o * rsqrt(mean(o^2) + eps)) * silu(z) ), o = bf16(gdn output)
 * z, y : bf16 [B, T, HV, DV];  norm_w : bf16 [DV].
 * Replaces the prefill + gated_rmsnorm plugin pair
 * (kernels/chunk_delta_cuda.h:46 followed by gatedRmsNormKernel.h:16 /
 * the TRT plugin gated_rmsnorm v1, gatedRmsNormPlugin.cpp:36-42). */
cudaError_t deltanet_chunk_prefill_gated(
    const void* q, const void* k, const void* v,
    const float* g, const float* beta,
    const void* z, const void* norm_w, float eps,
    void* y,
    const float* initial_state,
    float* final_state,
    int B, int T, int HV, int HQK, int DK, int DV, int chunk_size,
    void* workspace, size_t workspace_bytes,
    cudaStream_t stream);

/* Packed variable-length prefill: B = 1, T = total tokens, N sequences at
 * int32 offsets cu_seqlens[0..N] (cu_seqlens[0] = 0, non-decreasing,
 * cu_seqlens[N] = T). Each sequence starts from initial_states[i] (or zeros)
 * and writes final_states[i] ([N, HV, DK, DV] fp32). If z and norm_w are both
 * non-NULL the gated RMSNorm is fused and `out` receives y, else `out` receives o.
 * No counterpart in the reference, whose adapter is exact-T and ignores
 * context_lengths (gdnChunkPrefillSm87.h:16-19). */
cudaError_t deltanet_chunk_prefill_varlen(
    const void* q, const void* k, const void* v,
    const float* g, const float* beta,
    const void* z, const void* norm_w, float eps,
    void* out,
    const float* initial_states,
    float* final_states,
    const int* cu_seqlens, int N,
    int T, int HV, int HQK, int DK, int DV, int chunk_size,
    void* workspace, size_t workspace_bytes,
    cudaStream_t stream);

/* Long sequences in segments; no counterpart in the reference (its state carry
 * walks every chunk of a sequence in one serial loop, kernels/chunk_delta_cuda.cu:312-424).
 * Same inputs, outputs and results as deltanet_chunk_prefill (z and norm_w NULL:
 * `out` receives o) or deltanet_chunk_prefill_gated (both set: `out` receives y),
 * for few long sequences, where one pass leaves most of the GPU idle on the serial
 * chunk recurrence. Each sequence is cut at chunk boundaries into `segments`
 * segments (0: chosen for the current device from a wave model, 1 or a full GPU:
 * one pass) and three launches run on `stream`: every segment from a zero state
 * and from the identity with v = 0 (final states A_j and Phi_j, one grid), the
 * scan S_0 = initial_state, S_{j+1} = Phi_j S_j + A_j of the segments' entry
 * states, and every segment from its entry state (the output, and the final
 * state of the last segment). The passes run one CTA per (segment, head) or a
 * 4-CTA cluster per (segment, head), whichever the wave model finds cheaper
 * (GDN_B200_KERNEL=fused|split restricts the choice). The workspace must hold
 * deltanet_segmented_workspace_size(...) bytes for the same arguments and device
 * (256 when one pass is chosen). deltanet_segmented_plan reports the choice:
 * segments per sequence, chunks per segment, kernel (0: one pass, the plain call;
 * 1: one CTA per (segment, head); 2: cluster split). */
size_t deltanet_segmented_workspace_size(int B, int T, int HV, int DK, int DV, int chunk_size, int segments);
cudaError_t deltanet_segmented_plan(int B, int T, int HV, int segments, int* nseg, int* chunks_per_segment,
                                    int* kernel);
cudaError_t deltanet_chunk_prefill_segmented(
    const void* q, const void* k, const void* v,
    const float* g, const float* beta,
    const void* z, const void* norm_w, float eps,
    void* out,
    const float* initial_state,
    float* final_state,
    int B, int T, int HV, int HQK, int DK, int DV, int chunk_size, int segments,
    void* workspace, size_t workspace_bytes,
    cudaStream_t stream);

/* Inputs of the reference's TRT prefill adapter: the GDNParams fields that
 * runGdnChunkPrefillSm87 reads (gdnChunkPrefillSm87.cu:188-230), plus an
 * optional fused gated RMSNorm and the workspace. */
typedef struct gdn_prefill_params {
    const void* q;        /* fp16 [n, seq_len, h, k_dim], not normalised */
    const void* k;        /* fp16 [n, seq_len, h, k_dim], not normalised */
    const void* v;        /* fp16 [n, seq_len, hv, v_dim] */
    const void* a;        /* fp16 [n, seq_len, hv]  (decay pre-activation) */
    const void* b;        /* fp16 [n, seq_len, hv]  (beta pre-activation) */
    const float* A_log;   /* fp32 [hv] */
    const void* dt_bias;  /* fp16 [hv] */
    float* h0_source;     /* fp32 [n, hv, k_dim, v_dim]: initial state in, final state out (in place) */
    void* o;              /* fp16 [n, seq_len, hv, v_dim] out (y when z and norm_w are set) */
    const void* z;        /* optional fp16 [n, seq_len, hv, v_dim]: fuse the gated RMSNorm */
    const void* norm_w;   /* optional fp16 [v_dim] */
    float eps;            /* norm epsilon (used with z) */
    int n, seq_len, h, hv, k_dim, v_dim;
    void* workspace;      /* >= deltanet_prefill_workspace_size(...) bytes, device memory */
    size_t workspace_bytes;
} gdn_prefill_params;

/* One GDN prefill with the adapter's pre-stage fused into the kernel's load
 * path: q/k L2-normalised in fp32 (eps 1e-6) and rounded to bf16, v rounded to
 * bf16, g = -exp(A_log) * softplus(a + dt_bias) and beta = sigmoid(b) in fp32,
 * output o rounded to bf16 then stored as fp16, final state written back into
 * h0_source. Replaces runGdnChunkPrefillSm87 (gdnChunkPrefillSm87.h:21) and its
 * four pre-stage / conversion kernels and state copy-back
 * (gdnChunkPrefillSm87.cu:44-125, 246-313) with one launch. Returns 0 on
 * success, -1 (with a message on stderr) on failure, as the reference. */
int gdn_run_chunk_prefill(const gdn_prefill_params* params, cudaStream_t stream);

/* Decode form: T tokens per sequence processed one after another against
 * `state` ([B, HV, DK, DV] fp32, read and updated in place), with the same
 * q/k/v/g/beta layouts as the prefill and an optional fused gated RMSNorm
 * (z and norm_w both set: out receives y, else o). Per token:
 *   S <- S e^{g}; kv = S^T k; delta = (v - kv) beta; S <- S + k delta^T; o = S^T q / sqrt(DK).
 * Continues a prefill: passing its final state gives the same outputs as a
 * longer prefill. No counterpart in the reference, which leaves decode to stock
 * Edge-LLM (export/patches/orin_text_engine/README.md:15); the semantics are
 * transformers' torch_recurrent_gated_delta_rule. */
cudaError_t deltanet_recurrent_decode(
    const void* q, const void* k, const void* v,
    const float* g, const float* beta,
    const void* z, const void* norm_w, float eps,
    void* out, float* state,
    int B, int T, int HV, int HQK, int DK, int DV,
    cudaStream_t stream);

/* Standalone gated RMSNorm over rows of dv: y = w * round(o * rsqrt(mean(o^2)+eps)) * silu(z).
 * dtype 0 = fp16 I/O (the reference plugin's only format,
 * gatedRmsNormPlugin.cpp:155-167), 1 = bf16 I/O. Replaces
 * kernel::gatedRmsNormForward, gatedRmsNormKernel.h:16. */
cudaError_t gated_rmsnorm_forward(const void* o, const void* z, const void* w, void* y,
                                  int64_t rows, int dv, float eps, int dtype, cudaStream_t stream);

/* No counterpart in the reference. For callers that cannot allocate device
 * memory at call time (an inference engine's enqueue path that forbids
 * cudaMalloc, a real-time loop where an allocation would synchronise the
 * device): deltanet_chunk_prefill_gated with its scratch (the bounded-wait
 * status word) in a static device array of at most 256 bytes held by every GPU
 * that loads the library, instead of a workspace argument. Inputs and outputs
 * are still the caller's. Allocates nothing. Returns cudaErrorInvalidValue if a
 * call would need more scratch than the array holds. The first call on a device
 * looks up the array's address (make it before any stream capture). All calls
 * share the array and its last contents; calls that overlap on the GPU race on
 * it. */
cudaError_t deltanet_chunk_prefill_gated_noalloc(
    const void* q, const void* k, const void* v,
    const float* g, const float* beta,
    const void* z, const void* norm_w, float eps,
    void* y,
    const float* initial_state,
    float* final_state,
    int B, int T, int HV, int HQK, int DK, int DV, int chunk_size,
    cudaStream_t stream);

/* No counterpart in the reference. The status word of
 * deltanet_chunk_prefill_gated_noalloc's static scratch on the current device
 * (the caller of that entry has no workspace to pass to deltanet_read_status):
 * copied to *status_host after the work queued on `stream` (synchronises
 * `stream`); 0 = clean, bit 0 = a bounded wait timed out; cleared when
 * clear != 0. Allocates nothing. */
cudaError_t deltanet_noalloc_read_status(int* status_host, int clear, cudaStream_t stream);

/* Copy the device status word of a workspace to *status_host (synchronises
 * `stream`). 0 = clean; bit 0 = a bounded wait timed out (each wait gives up
 * after about 1 s). The bits above say which part gave up: 8-11 the
 * cluster-split kernel's chain CTA (compute warps, MMA warp, load warp, output
 * MMA warp), 12-13 its prep CTAs (compute warps, gate warp), 14 its output CTA,
 * 15 the one-CTA-per-head kernel. Clears it when clear != 0. No counterpart in
 * the reference (its kernels have no waits). */
cudaError_t deltanet_read_status(void* workspace, int* status_host, int clear, cudaStream_t stream);

/* Test hook for failure detection; no counterpart in the reference (its
 * kernels have no waits; its error convention is the return code,
 * kernels/chunk_delta_cuda.cu:706-727). Runs deltanet_chunk_prefill_gated with
 * the v-tile load of chunk `withheld_chunk` never issued, so that the kernel's
 * bounded wait for that tile runs out (about 1 s): the kernel sets bit 0 of
 * the workspace status word (and the bit of the role that gave up, see
 * deltanet_read_status), stops its loop, waits (bounded) for the copies and
 * MMAs it has in flight, frees its tensor memory and returns; y and
 * final_state are then undefined. kernel: 0 = the launcher's choice, 1 = one
 * CTA per (sequence, v-head), 2 = the cluster-split kernel
 * (cudaErrorNotSupported if it cannot run). Returns the launch status. */
cudaError_t deltanet_test_withheld_load(
    const void* q, const void* k, const void* v,
    const float* g, const float* beta,
    const void* z, const void* norm_w, float eps,
    void* y,
    const float* initial_state,
    float* final_state,
    int B, int T, int HV, int HQK, int DK, int DV, int chunk_size,
    void* workspace, size_t workspace_bytes,
    cudaStream_t stream, int kernel, int withheld_chunk);

/* Library build identifier (for logs and tests). */
const char* gdn_b200_version(void);

#ifdef __cplusplus
}
#endif

#endif /* GDN_B200_GDN_PREFILL_H_ */
