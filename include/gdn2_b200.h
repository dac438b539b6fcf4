/*
 * gdn2_b200.h -- C ABI of the B200 GatedDeltaNet2 (GDN-2) core-recurrence library.
 *
 * The library (libgdn2_b200.so, built for sm_100a) replaces the Triton/FLA
 * kernels behind the GDN-2 token mixer of Gabz4200/QwenDopamine:
 *   - chunkwise forward   chunk_gdn2 / chunk_gdn2_fwd
 *                         (src/qwendopamine/models/gdn2/gdn2_ops/chunk_gdn2.py:1165-1434)
 *   - chunkwise backward  ChunkGDN2Function.backward / chunk_gdn2_bwd
 *                         (chunk_gdn2.py:2170-2325, 2461-2547)
 *   - recurrent decode    fused_recurrent_gdn2 / fused_recurrent_gdn2_fwd
 *                         (gdn2_ops/fused_recurrent_gdn2.py:344-555)
 *   - context-parallel pre-scan and merge (the FLA-CP algorithm of
 *                         gdn2_ops/chunk_kda.py:182-1299, applied to GDN-2)
 *
 * Conventions
 *   - Every pointer is device memory unless stated otherwise; the caller owns
 *     all allocations (sizes come from the *_bytes queries below).
 *   - Token tensors are contiguous [rows, H, D] where rows = B*T (fixed length)
 *     or the packed token count (varlen, batch 1).  Sequence n owns rows
 *     [cu_seqlens[n], cu_seqlens[n+1]) and is cut into chunks of 64 rows.
 *   - Recurrent states are fp32, contiguous [N, H, K, V] (key-major).
 *   - Every entry point returns GDN2_OK (0) or an error code; after an error,
 *     gdn2_last_error() returns a message for the calling thread.
 *   - Work is enqueued on `stream` (a cudaStream_t passed as void*); calls are
 *     asynchronous with respect to the host.
 */
#ifndef GDN2_B200_H
#define GDN2_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element types of token tensors */
enum {
    GDN2_DTYPE_F32 = 0,
    GDN2_DTYPE_BF16 = 1,
    GDN2_DTYPE_F16 = 2
};

/* status codes */
enum {
    GDN2_OK = 0,
    GDN2_ERR_INVALID = 1,     /* bad argument: shape, dtype, null pointer, size */
    GDN2_ERR_UNSUPPORTED = 2, /* valid but not implemented (e.g. K > 256)       */
    GDN2_ERR_CUDA = 3,        /* a CUDA runtime call failed                     */
    GDN2_ERR_WORKSPACE = 4    /* caller-provided buffer too small               */
};

/* Sequence / chunk geometry shared by the chunkwise entry points.
 * cu_seqlens[N+1] (token offsets), chunk_offsets[N+1] (chunk offsets,
 * chunk_offsets[n+1]-chunk_offsets[n] = ceil(len_n/64)) and chunk_seq[n_chunks]
 * (owning sequence of each chunk) are int32 device arrays; the Python layer
 * builds them the way prepare_chunk_indices does (chunk_gdn2.py:1385-1389). */
typedef struct gdn2_seqs {
    int64_t total_tokens;
    int32_t n_seqs;
    int32_t n_chunks;
    const int32_t* cu_seqlens;
    const int32_t* chunk_offsets;
    const int32_t* chunk_seq;
} gdn2_seqs;

/* A chunkwise problem: q,k,g,b are [rows,H,K]; v,w,o are [rows,H,V].
 * g (and dg) are always fp32 (the module's fp32_decay=True default,
 * gdn2.py:840-845); q,k,v,b,w,o and their gradients share `dtype`.
 * Gate in kernel (use_gate_in_kernel, chunk_gdn2.py:1194-1204, 2316-2323;
 * bf16 problems with K and V multiples of 8 only): gate = 1 reads g as the raw
 * pre-activation and uses -exp(A_log[h]) * softplus(g + dt_bias[h][k]) as the
 * log-decay, gate = 2 uses lower_bound * sigmoid(exp(A_log[h]) * (g +
 * dt_bias[h][k])); A_log fp32 [H], dt_bias fp32 [H*K] or NULL.  The backward
 * then returns dg for the raw input and ADDS dL/dA_log into dA_log [H] and
 * dL/d dt_bias into ddt_bias [H*K] (fp32; the caller zeroes them). */
typedef struct gdn2_chunk_problem {
    int32_t H, K, V;
    int32_t dtype;
    int32_t use_qk_l2norm; /* use_qk_l2norm_in_kernel (chunk_gdn2.py:1283) */
    float scale;           /* defaults to K**-0.5 on the Python side        */
    gdn2_seqs seqs;
    const float* A_log;
    const float* dt_bias;
    int32_t gate;          /* 0: g is the log-decay; 1, 2: gate in kernel   */
    float lower_bound;
    float* dA_log;
    float* ddt_bias;
    /* SM budget of one launch; 0 = the whole GPU.  No counterpart in the
     * reference: a caller that runs a state pass and an intra-chunk kernel
     * on two streams at the same time divides the SMs between them this way.
     *   - gdn2_chunk_fwd_intra (bf16, head sizes up to 128): the persistent
     *     kernel launches at most max_ctas CTAs (one per SM otherwise);
     *   - gdn2_chunk_fwd_state / gdn2_chunk_bwd_state (bf16, K = V = 128):
     *     the split of each sequence-head's value columns over two CTAs is
     *     used only while it stays within max_ctas CTAs; otherwise one CTA
     *     per sequence-head walks the whole state. */
    int32_t max_ctas;
} gdn2_chunk_problem;

/* ---- library information ------------------------------------------------ */
const char* gdn2_version(void);
const char* gdn2_status_string(int status);
const char* gdn2_last_error(void);

/* ---- chunkwise forward ---------------------------------------------------
 * Replaces chunk_gdn2_fwd (chunk_gdn2.py:1165-1264) and its kernels K1-K7
 * (intra-chunk scores, WY inverse, w/u recompute, inter-chunk state pass and
 * output).  `saved` receives the per-chunk intermediates the backward needs
 * (the ctx.save_for_backward set of chunk_gdn2.py:2425-2448, in B200 layout);
 * its size is gdn2_chunk_saved_bytes().  h0 / ht may be NULL (zero initial
 * state / no final state).  The two phases are also exported separately so a
 * context-parallel caller can run the pre-scan between them. */
size_t gdn2_chunk_saved_bytes(const gdn2_chunk_problem* p);
int gdn2_chunk_fwd(const gdn2_chunk_problem* p,
                   const void* q, const void* k, const void* v, const float* g,
                   const void* b, const void* w, const float* h0,
                   void* o, float* ht, void* saved, size_t saved_bytes,
                   void* stream);
/* phase 1: intra-chunk solve (fully parallel over chunks and heads) */
int gdn2_chunk_fwd_intra(const gdn2_chunk_problem* p,
                         const void* q, const void* k, const void* v, const float* g,
                         const void* b, const void* w,
                         void* saved, size_t saved_bytes, void* stream);
/* phase 2: inter-chunk state pass with fused output (sequential over chunks) */
int gdn2_chunk_fwd_state(const gdn2_chunk_problem* p, const float* h0,
                         void* o, float* ht, void* saved, size_t saved_bytes,
                         void* stream);

/* ---- chunkwise backward --------------------------------------------------
 * Replaces chunk_gdn2_bwd (chunk_gdn2.py:2170-2325): reverse state pass
 * (K10), dq/dk/dv/db/dw/dg (K9, K11, K12, K13) and the l2norm backward.
 * dht / dh0 / h0 may be NULL.  `workspace` is gdn2_chunk_bwd_workspace_bytes(). */
size_t gdn2_chunk_bwd_workspace_bytes(const gdn2_chunk_problem* p);
int gdn2_chunk_bwd(const gdn2_chunk_problem* p,
                   const void* q, const void* k, const void* v, const float* g,
                   const void* b, const void* w,
                   const void* saved, size_t saved_bytes,
                   const void* dout, const float* dht,
                   void* dq, void* dk, void* dv, float* dg, void* db, void* dw,
                   float* dh0, void* workspace, size_t workspace_bytes,
                   void* stream);

/* phase 1: reverse state pass (sequential over chunks); fills `workspace`
 * with the per-chunk state gradients and dVN, writes dh0 when non-NULL */
int gdn2_chunk_bwd_state(const gdn2_chunk_problem* p, const void* saved,
                         size_t saved_bytes, const void* dout, const float* dht,
                         float* dh0, void* workspace, size_t workspace_bytes,
                         void* stream);
/* phase 2: per-chunk gradients (fully parallel over chunks and heads); reads
 * what phase 1 left in `workspace` (and, for heads above 128 channels, uses a
 * further section of it as scratch) */
int gdn2_chunk_bwd_intra(const gdn2_chunk_problem* p,
                         const void* q, const void* k, const void* v, const float* g,
                         const void* b, const void* w,
                         const void* saved, size_t saved_bytes, const void* dout,
                         void* dq, void* dk, void* dv, float* dg, void* db, void* dw,
                         void* workspace, size_t workspace_bytes, void* stream);

/* ---- chunkwise backward without allocation -------------------------------
 * No counterpart in the reference.  gdn2_chunk_bwd with its workspace taken
 * from a scratch array built into the library (GDN2_NOALLOC_SCRATCH_BYTES per
 * GPU, held until the process exits) instead of from the caller.  For callers
 * that cannot allocate device memory while they run the backward: a plugin
 * host that owns all device memory and hands an op only its inputs and
 * outputs, or a loop that has reserved nearly all HBM and must not risk an
 * allocation failure or the device synchronisation cudaMalloc/cudaFree can
 * cause mid-step.  It allocates nothing itself.
 *   - Problems whose gdn2_chunk_bwd_workspace_bytes() exceeds the built-in
 *     size are rejected with GDN2_ERR_WORKSPACE (the message gives both sizes).
 *   - The first call on a device (with that device current) looks up the
 *     array's device address once; make it before any stream capture.  The
 *     address stays cached for the process's life, so do not call this again
 *     on a device after cudaDeviceReset (its primary context is re-created).
 *   - All calls on a device share the array and leave their data in it;
 *     nothing needs to start at zero.  Calls that overlap on the GPU race:
 *     order them (one stream, or events). */
#define GDN2_NOALLOC_SCRATCH_BYTES (32u << 20)
int gdn2_chunk_bwd_noalloc(const gdn2_chunk_problem* p,
                           const void* q, const void* k, const void* v, const float* g,
                           const void* b, const void* w,
                           const void* saved, size_t saved_bytes,
                           const void* dout, const float* dht,
                           void* dq, void* dk, void* dv, float* dg, void* db, void* dw,
                           float* dh0, void* stream);

/* ---- recurrent (decode) forward ------------------------------------------
 * Replaces fused_recurrent_gdn2_fwd (fused_recurrent_gdn2.py:344-458) and its
 * kernel (:117-341).  q,k: [B,T,H,K]; v,w: [B,T,HV,V]; g,b: [B,T,HV,K]
 * (HV a multiple of H: grouped value heads).  With cu_seqlens (int32 [N+1],
 * B == 1) sequences are packed.  With state_indices (int32 [N]) h0 and ht are
 * state pools indexed per sequence (slot stride state_stride elements) and
 * the update is in place; otherwise h0 / ht are [N,HV,K,V] and ht may equal h0
 * for an in-place update.  h0 == NULL means zero state; ht == NULL means the
 * final state is not stored.
 * Speculative decoding (fused_recurrent_gdn2.py:217-226, 311-324): with
 * state_indices_stride > 0, state_indices is [N, state_indices_stride]; the
 * sequence starts from slot state_indices[n][a-1] (a = num_accepted_tokens[n],
 * or 1 when num_accepted_tokens is NULL) and the state after its token t is
 * written to slot state_indices[n][t] of ht (the pool, normally == h0).
 * Negative slots are skipped (a negative starting slot skips the sequence).
 * With state_indices_stride == 0 the indices are [N] and only the final state
 * is written, to slot state_indices[n].
 * Gate in kernel (fused_recurrent_gdn2.py:257-272): gate = 0 takes g as the
 * log-decay; gate = 1 uses -exp(A_log[h]) * softplus(g + dt_bias[h][k]) and
 * gate = 2 uses lower_bound * sigmoid(exp(A_log[h]) * (g + dt_bias[h][k])),
 * h the key head of the value head (A_log fp32 [H], dt_bias fp32 [H*K] or
 * NULL). */
typedef struct gdn2_recurrent_problem {
    int32_t B, T, H, HV, K, V;
    int32_t dtype;
    int32_t use_qk_l2norm;
    float scale;
    int32_t n_seqs;
    const int32_t* cu_seqlens;
    const int32_t* state_indices;
    int64_t state_stride;
    int64_t state_indices_stride;
    const int32_t* num_accepted_tokens;
    const float* A_log;
    const float* dt_bias;
    int32_t gate;
    float lower_bound;
} gdn2_recurrent_problem;

int gdn2_recurrent_fwd(const gdn2_recurrent_problem* p,
                       const void* q, const void* k, const void* v, const float* g,
                       const void* b, const void* w, const float* h0,
                       void* o, float* ht, void* stream);

/* ---- context parallelism (sequence-parallel long context) ----------------
 * Each rank owns a contiguous span of whole chunks of one sequence set.
 * Forward: after gdn2_chunk_fwd_intra, gdn2_cp_fwd_prescan writes this rank's
 * affine span map  S_out = M S_in + h_e  as hm = [N,H,K,V+K] fp32
 * (h_e in columns [0,V), M in columns [V,V+K)), the message that FLA-CP
 * all-gathers (chunk_kda.py:1101-1185).  After the all-gather, gdn2_cp_merge
 * folds the maps of ranks 0..rank-1 into this rank's initial state
 * (chunk_kda.py:509-697, FORWARD=True).
 * Backward: gdn2_cp_bwd_prescan writes dhm = [N,H,K,V], the state gradient
 * this span's outputs (and `dht`, the gradient of its end state if that is
 * the sequence's final state; NULL otherwise) produce at the span's start; gdn2_cp_merge with forward=0 folds
 * ranks world-1..rank+1 (using their forward M, transposed) into this rank's
 * dht.  `hm_all` is [world, N, H, K, V+K] and `dhm_all` is [world, N, H, K, V]
 * (rank-major, the layout all_gather_into_tensor produces).
 *   forward=1:  x = init (or 0);  for j = 0 .. rank-1:        x = M_j x + h_e_j
 *   forward=0:  x = init (or 0);  for j = world-1 .. rank+1:  x = M_j^T x + dhm_j
 * and state_out = x ([N,H,K,V] fp32).  `init` is the global initial state
 * (forward) or the gradient of the global final state (backward).
 * Workspace: gdn2_cp_workspace_bytes(p) is 0 or the size of a buffer that
 * lets gdn2_cp_bwd_prescan run the tensor-core backward state pass (bf16,
 * K = V = 128); given one at least that large (a gdn2_chunk_bwd workspace
 * is), the pre-scan writes scratch tiles into it, otherwise it runs the
 * register-state pass.  gdn2_cp_fwd_prescan takes no workspace (pass NULL). */
size_t gdn2_cp_workspace_bytes(const gdn2_chunk_problem* p);
int gdn2_cp_fwd_prescan(const gdn2_chunk_problem* p, const void* saved,
                        size_t saved_bytes, float* hm, void* workspace,
                        size_t workspace_bytes, void* stream);
int gdn2_cp_bwd_prescan(const gdn2_chunk_problem* p, const void* saved,
                        size_t saved_bytes, const void* dout, const float* dht,
                        float* dhm, void* workspace, size_t workspace_bytes,
                        void* stream);
int gdn2_cp_merge(const gdn2_chunk_problem* p, const float* hm_all,
                  const float* dhm_all, int32_t rank, int32_t world,
                  int32_t forward, const float* init, float* state_out,
                  void* stream);
/* The same folds over the n_sub consecutive sub-spans of one span, keeping
 * every intermediate (the chunk_kda.py:509-697 merge run as a scan): with
 * hm_sub [n_sub, N, H, K, V+K] and dhm_sub [n_sub, N, H, K, V] (sub-span
 * major) it writes states [n_sub, N, H, K, V]:
 *   forward=1:  states[0] = init;  states[s+1] = M_s states[s] + h_e_s
 *   forward=0:  states[n_sub-1] = init;  states[s] = M_{s+1}^T states[s+1] + dhm_{s+1}
 * i.e. the start state (end-state gradient) of every sub-span.  K <= 128 (a
 * multiple of 16), V a multiple of 4; GDN2_ERR_UNSUPPORTED otherwise. */
int gdn2_cp_unfold(const gdn2_chunk_problem* p, const float* hm_sub,
                   const float* dhm_sub, int32_t n_sub, int32_t forward,
                   const float* init, float* states, void* stream);

/* ---- block prologue / epilogue -------------------------------------------
 * Causal depthwise convolution with optional SiLU, one per q / k / v
 * projection (ShortConvolution, gdn2.py:372-430), over x [B][T][D]:
 *   c[b,t,d] = round(bias[d] + sum_{j<W} weight[d][j] * x[b, t-W+1+j, d])
 *   y[b,t,d] = silu(c) (activation 1) or c (activation 0), rounded
 * round() is the token dtype's rounding: the reference's convolution output
 * is in that dtype before its activation.  Rows before t = 0 come from
 * `prefix` (W-1 rows per batch entry; element (b, i, d) at prefix[b*sb +
 * i*sw + d*sd]; the previous span's last tokens under sequence parallelism,
 * or a decode cache [B][D][W-1] through its strides) or are zero when NULL.
 * weight [D][W] and bias [D] (or NULL) are fp32 copies of the parameters.
 * new_state (or NULL) receives the last W-1 rows of [prefix; x] as
 * [B][D][W-1] (the reference's conv cache layout).  D % 8 == 0, W <= 4, and
 * x / y / dy / dx start on 16-byte boundaries. */
typedef struct gdn2_conv_problem {
    int32_t B, T, D, W;
    int32_t dtype;
    int32_t activation;          /* 0: none, 1: silu */
    int64_t prefix_sb, prefix_sw, prefix_sd;  /* element strides of prefix */
} gdn2_conv_problem;

int gdn2_conv_fwd(const gdn2_conv_problem* p, const void* x, const float* weight,
                  const float* bias, const void* prefix, void* y, void* new_state,
                  void* stream);
/* Backward: dx [B][T][D] (token dtype); dweight [D][W] and dbias [D] (or
 * NULL) fp32, written; dprefix (or NULL) fp32 [B][W-1][D] contiguous, the
 * gradient of the prefix rows (sent back to the previous span's owner under
 * sequence parallelism).  Deterministic: per-block partial sums go through
 * `workspace` and are reduced in a fixed order. */
size_t gdn2_conv_bwd_workspace_bytes(const gdn2_conv_problem* p);
int gdn2_conv_bwd(const gdn2_conv_problem* p, const void* x, const float* weight,
                  const float* bias, const void* prefix, const void* dy, void* dx,
                  float* dweight, float* dbias, float* dprefix, void* workspace,
                  size_t workspace_bytes, void* stream);

/* SiLU-gated RMSNorm of the block epilogue (RMSNormGated, gdn2.py:433-452)
 * over the last dimension N of x, z [rows][N]:
 *   y = x * rsqrt(mean(x^2) + eps) * weight * silu(z)
 * evaluated as the reference does, in the input dtype: every intermediate
 * (x^2, the mean, mean + eps, its rsqrt, the products, silu(z)) is rounded
 * to `dtype`; a product with an fp32 weight is fp32, and y has the promoted
 * type (dtype, weight_dtype).  weight_dtype is `dtype` or fp32.  With
 * fp32_math = 1 (the reference under torch.autocast, where pow and rsqrt run
 * in fp32): x^2, the mean, rsqrt and every product stay fp32, silu(z) is
 * still rounded to `dtype`, and y is fp32 (weight_dtype must be fp32).
 * N % 8 == 0 and N <= 256. */
typedef struct gdn2_norm_problem {
    int64_t rows;
    int32_t N;
    int32_t dtype;          /* x, z, dx, dz */
    int32_t weight_dtype;   /* weight; dy and y have the promoted type */
    float eps;
    int32_t fp32_math;
} gdn2_norm_problem;

int gdn2_gated_norm_fwd(const gdn2_norm_problem* p, const void* x, const void* z,
                        const void* weight, void* y, void* stream);
/* Backward (fp32 arithmetic): dx, dz in `dtype`; dweight fp32 [N], written. */
size_t gdn2_gated_norm_bwd_workspace_bytes(const gdn2_norm_problem* p);
int gdn2_gated_norm_bwd(const gdn2_norm_problem* p, const void* x, const void* z,
                        const void* weight, const void* dy, void* dx, void* dz,
                        float* dweight, void* workspace, size_t workspace_bytes,
                        void* stream);

/* Device-side fault bits.  Kernels that wait on asynchronous copies or on
 * tensor-core completion bound every wait in time (about one second); a wait
 * that runs out makes the kernel release its tensor memory, return without
 * finishing, and set a bit of a per-device fault word (bit 0: state passes,
 * bit 1: forward intra-chunk kernel, bit 2: decode, bit 3: backward
 * intra-chunk kernel).  gdn2_fault_status
 * synchronises `stream` (the default stream when NULL), returns the fault
 * word of the current device (0 = no fault) and resets it when `clear` is
 * nonzero; a negative return is a CUDA error.  No counterpart in the
 * reference, whose kernels contain no bounded waits. */
int gdn2_fault_status(void* stream, int32_t clear);

/* ---- test hook: the bounded-wait abort path ---------------------------------
 * No counterpart in the reference.  Runs the forward state pass
 * (gdn2_chunk_fwd_state, no initial or final state) with chunk `skip_chunk`'s
 * tiles never requested and every wait limited to `wait_ns` nanoseconds
 * (1 .. 1e9), so that the wait for that chunk runs out: the kernel drains its
 * copies and products in flight, frees its tensor memory, sets bit 0 of the
 * fault word and returns.  Nothing faults and nothing waits without a limit;
 * the context stays usable and gdn2_fault_status(stream, 1) reports the bit.
 * Only problems the tcgen05 state pass serves (bf16, K = V = 128) are
 * accepted (GDN2_ERR_UNSUPPORTED otherwise).  The outputs are incomplete: a
 * test of the failure path, not a compute entry point. */
int gdn2_test_fwd_state_wait_timeout(const gdn2_chunk_problem* p, void* o, void* saved,
                                     size_t saved_bytes, int32_t skip_chunk, uint64_t wait_ns,
                                     void* stream);

#ifdef __cplusplus
}
#endif
#endif /* GDN2_B200_H */
