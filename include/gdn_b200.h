/*
 * gdn_b200.h — C ABI of the B200 (sm_100a) Gated DeltaNet token mixer.
 *
 * This library replaces the call
 *     o, final_state = chunk_gated_delta_rule(q, k, v, g, beta, scale=..., initial_state=...,
 *                                             output_final_state=..., use_qk_l2norm_in_kernel=...,
 *                                             cu_seqlens=..., cu_seqlens_cpu=...)
 * made by soreRNN at sore/model/gdn.py:166-169 (flash-linear-attention's Triton op,
 * fla/ops/gated_delta_rule/chunk.py:365-380, with its autograd backward at chunk.py:117-236),
 * and adds the single-token decode step (the API shape of fla's fused_recurrent_gated_delta_rule,
 * fla/ops/gated_delta_rule/fused_recurrent.py:291-308) and the per-segment affine state map used to
 * split a long prefill by sequence across GPUs.
 *
 * Math (soreRNN sore/model/gdn_ref.py:17-21), per sequence n and value head h, state S [DK, DV]:
 *     S <- exp(g_t) S ;  delta = beta_t (v_t - S^T k_t) ;  S <- S + k_t delta^T ;  o_t = scale S^T q_t
 * Value head h reads q/k head h / (HV / H) (grouped value attention, gdn.py:153-156).
 *
 * Conventions of every entry point:
 *  - all pointers are device pointers unless named *_host; tensors are C-contiguous:
 *      q, k, dq, dk      [B, T, H,  DK]        (dtype: act_dtype)
 *      v, o, do, dv      [B, T, HV, DV]        (dtype: act_dtype)
 *      g, dg             [B, T, HV]            (g: g_dtype; dg: fp32)
 *      beta, dbeta       [B, T, HV]            (beta: beta_dtype; dbeta: fp32)
 *      states            [N, HV, DK, DV] fp32  (initial_state, final_state, dh0, dht)
 *    With cu_seqlens (int64 [N+1], device) B must be 1 and the state restarts at every
 *    cu_seqlens[i] (gdn_ref.py:53-61); without it every batch row is one sequence (N = B).
 *  - the caller allocates every output and the workspace (size from the *_workspace_size query);
 *    the library never allocates device memory. Its only device state: one 4-byte error word per
 *    workspace-less streaming kernel family (decode, norm-gate, conv; see gdn_stream_kernels_error)
 *    and the fixed scratch array of gdn_chunk_bwd_noalloc.
 *  - every call is stream-ordered on `stream`, does not synchronise the host, and returns a status
 *    code (GDN_OK = 0); nothing aborts or traps. Shapes, dtypes and alignment are checked on the host
 *    before any launch.
 */
#ifndef GDN_B200_H
#define GDN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* gdn_stream_t; /* same object as cudaStream_t */

enum gdn_status {
    GDN_OK = 0,
    GDN_ERR_SHAPE = 1,       /* inconsistent or unsupported sizes */
    GDN_ERR_DTYPE = 2,       /* unsupported dtype code */
    GDN_ERR_ALIGN = 3,       /* pointer not aligned as the kernel needs (16 B) */
    GDN_ERR_LAUNCH = 4,      /* a CUDA launch or tensor-map encode failed */
    GDN_ERR_TIMEOUT = 5,     /* a device-side bounded wait ran out (see gdn_workspace_error) */
    GDN_ERR_WORKSPACE = 6,   /* workspace pointer NULL or smaller than the query said */
    GDN_ERR_ARGUMENT = 7,    /* NULL pointer for a required tensor, bad flag */
    GDN_ERR_SCRATCH_LIMIT = 8 /* problem needs more scratch than gdn_chunk_bwd_noalloc's fixed array */
};

enum gdn_dtype { GDN_BF16 = 0, GDN_FP16 = 1, GDN_FP32 = 2 };

/* Problem description shared by the chunked forward/backward entry points. */
typedef struct gdn_problem {
    int64_t B, T, H, HV, DK, DV;  /* see the layouts above */
    int64_t N;                    /* number of sequences: B, or len(cu_seqlens) - 1 */
    const int64_t* cu_seqlens;    /* device [N+1] or NULL */
    int64_t max_seqlen;           /* longest sequence (host-known, e.g. from cu_seqlens_cpu); <=0: B*T */
    float scale;                  /* o = scale * S^T q; the reference passes DK^-0.5 (gdn.py:148) */
    int32_t act_dtype;            /* dtype of q, k, v, o, do, dq, dk, dv */
    int32_t g_dtype;              /* dtype of g */
    int32_t beta_dtype;           /* dtype of beta */
    int32_t use_qk_l2norm;        /* 1: q, k are L2-normalised per head inside the kernel (gdn.py:168) */
    int32_t ckpt_every;           /* forward keeps one state checkpoint every this many 64-token chunks */
} gdn_problem;

/* Human-readable text for a status code (static storage). */
const char* gdn_status_string(int status);

/* Which kernel family a problem runs on: 1 = chunked tcgen05 (bf16, DK = DV = 128),
 * 0 = recurrent fp32-accumulating kernels (fp32 inputs, other head sizes). */
int gdn_uses_chunk_kernels(const gdn_problem* p);

/* Number of fp32 [HV, DK, DV] state checkpoints the forward writes for the backward
 * (an upper bound when cu_seqlens is given; computed from max_seqlen and N only). */
int64_t gdn_checkpoint_count(const gdn_problem* p);

/* Workspace bytes for gdn_chunk_fwd / gdn_chunk_bwd (0 is possible). */
size_t gdn_chunk_fwd_workspace_size(const gdn_problem* p);
size_t gdn_chunk_bwd_workspace_size(const gdn_problem* p);

/*
 * Forward: o = GDN(q, k, v, g, beta) from initial_state (NULL = zeros).
 * final_state (NULL = not wanted) receives S after the last token of each sequence.
 * checkpoints (NULL = not wanted; needed by gdn_chunk_bwd) receives gdn_checkpoint_count(p)
 * states [HV, DK, DV] fp32: the state at the start of chunk c of sequence n for c % ckpt_every == 0.
 * Replaces: fla chunk_gated_delta_rule forward (chunk.py:365-380, as called at gdn.py:166-169).
 */
int gdn_chunk_fwd(const gdn_problem* p, const void* q, const void* k, const void* v, const void* g,
                  const void* beta, const float* initial_state, void* o, float* final_state,
                  float* checkpoints, void* workspace, size_t workspace_bytes, gdn_stream_t stream);

/*
 * Backward of gdn_chunk_fwd given do (and dht = gradient of final_state, NULL = zero).
 * Recomputes every chunk state from the forward's checkpoints (nothing per chunk is stored by the
 * forward). dq, dk, dv are written in act_dtype; dg, dbeta in fp32; dh0 (NULL = not wanted) fp32.
 * Replaces: ChunkGatedDeltaRuleFunction.backward (fla chunk.py:117-236).
 */
int gdn_chunk_bwd(const gdn_problem* p, const void* q, const void* k, const void* v, const void* g,
                  const void* beta, const float* initial_state, const float* checkpoints, const void* dout,
                  const float* dht, void* dq, void* dk, void* dv, float* dg, float* dbeta, float* dh0,
                  void* workspace, size_t workspace_bytes, gdn_stream_t stream);

/*
 * Saved-record variant of the pair above, for problems with gdn_uses_chunk_kernels(p) == 1 (others get
 * GDN_ERR_SHAPE). gdn_chunk_fwd_save is gdn_chunk_fwd that, in place of the sparse checkpoints, also writes
 * the backward's per-(64-token chunk, value head) record into `saved` (gdn_chunk_saved_bytes(p) bytes,
 * 16-byte aligned; 88 KB per chunk-head, e.g. 704 MB for 8 x 4,096 tokens x 16 heads): the chunk-start
 * state S0^T, -W, T = (I + A)^-1, Delta^T and the low part of Dd^T, as bf16 operand tiles. Given those
 * records, gdn_chunk_bwd_saved (workspace: gdn_chunk_bwd_saved_workspace_size) runs the reverse sweep
 * without the recompute pass that gdn_chunk_bwd needs. Same results as the checkpoint pair within bf16
 * rounding of the records; the trade is memory held between the two calls for one pass less.
 * p->ckpt_every is not used by this pair but must be valid (>= 1). With cu_seqlens the buffer is sized for
 * the worst split of the tokens; the forward zeroes the slots past the last sequence's chunks.
 * Replaces: the same two calls as gdn_chunk_fwd / gdn_chunk_bwd (fla chunk.py:365-380, 117-236).
 */
size_t gdn_chunk_saved_bytes(const gdn_problem* p);
size_t gdn_chunk_bwd_saved_workspace_size(const gdn_problem* p);
int gdn_chunk_fwd_save(const gdn_problem* p, const void* q, const void* k, const void* v, const void* g,
                       const void* beta, const float* initial_state, void* o, float* final_state, void* saved,
                       void* workspace, size_t workspace_bytes, gdn_stream_t stream);
int gdn_chunk_bwd_saved(const gdn_problem* p, const void* q, const void* k, const void* v, const void* g,
                        const void* beta, const void* saved, const void* dout, const float* dht, void* dq, void* dk,
                        void* dv, float* dg, float* dbeta, float* dh0, void* workspace, size_t workspace_bytes,
                        gdn_stream_t stream);

/*
 * The state-gradient half of gdn_chunk_bwd_saved: dh0 (fp32 [N, HV, DK, DV], required) = the gradient of every
 * sequence's initial state given do and dht (NULL = zero), with no token gradients. The reverse sweep then
 * carries dS alone and skips the per-chunk gradient steps (about half of its work per chunk). Workspace:
 * gdn_chunk_bwd_saved_workspace_size(p) bytes. Used to join pieces of sequences (gdn_piece_chain): the
 * gradient each piece passes back from a zero end-state gradient.
 * Replaces: part of ChunkGatedDeltaRuleFunction.backward (fla chunk.py:117-236): its dh0 output alone.
 */
int gdn_chunk_state_grad_saved(const gdn_problem* p, const void* q, const void* k, const void* v, const void* g,
                               const void* beta, const void* saved, const void* dout, const float* dht, float* dh0,
                               void* workspace, size_t workspace_bytes, gdn_stream_t stream);

/* Size of gdn_chunk_bwd_noalloc's fixed scratch array (36 MiB). */
#define GDN_NOALLOC_SCRATCH_BYTES ((size_t)36 << 20)

/*
 * gdn_chunk_bwd for callers that cannot allocate device memory. No counterpart in the reference.
 * Some callers have no device allocator at call time: a host runtime reaching this library over a plain
 * C FFI without an allocator of its own, or a plugin whose execute hook must not allocate. This variant
 * takes gdn_chunk_bwd's arguments minus the workspace and allocates nothing (no cudaMalloc/cudaFree);
 * its scratch is one fixed array of GDN_NOALLOC_SCRATCH_BYTES inside the library's device image, held on
 * every GPU that loads the library until the process exits. Problems whose
 * gdn_chunk_bwd_workspace_size() exceeds it are rejected with GDN_ERR_SCRATCH_LIMIT before any launch;
 * invalid problems get gdn_chunk_bwd's status. With the chunked kernels the array holds 418 chunk-heads
 * (64-token chunks x value heads): e.g. T = 1,024 with 16 heads, or T = 4,096 with 6 heads, per call.
 * All calls on a device share the array: calls whose GPU work overlaps (other streams, other host
 * threads) race, so order them on one stream. Device-side timeouts are not reported (the error word is
 * in the array): use gdn_chunk_bwd + gdn_workspace_error for that. The first call on each device looks
 * the array's address up and keeps it for the life of the device's primary context; make that first
 * call before any stream capture begins.
 */
int gdn_chunk_bwd_noalloc(const gdn_problem* p, const void* q, const void* k, const void* v, const void* g,
                          const void* beta, const float* initial_state, const float* checkpoints,
                          const void* dout, const float* dht, void* dq, void* dk, void* dv, float* dg,
                          float* dbeta, float* dh0, gdn_stream_t stream);

/*
 * One decode token for N sequences on a resident fp32 state [N, HV, DK, DV], updated in place:
 * q, k [N, H, DK], v [N, HV, DV], g, beta [N, HV] (dtypes as in gdn_problem), o [N, HV, DV].
 * Math: one iteration of gdn_ref.py:18-21. Replaces: fla fused_recurrent_gated_delta_rule
 * (fused_recurrent.py:291-308) with T = 1, initial_state = state, output_final_state in place.
 */
int gdn_decode_step(int64_t N, int64_t H, int64_t HV, int64_t DK, int64_t DV, float scale,
                    int32_t act_dtype, int32_t g_dtype, int32_t beta_dtype, int32_t use_qk_l2norm,
                    const void* q, const void* k, const void* v, const void* g, const void* beta,
                    float* state, void* o, gdn_stream_t stream);

/*
 * The gate and beta activations the layer can hand to the mixer (sore/model/gdn.py:157-162:
 * use_gate_in_kernel=True, A_log, dt_bias, use_beta_sigmoid_in_kernel=True, with the raw a_proj / b_proj
 * outputs passed as g and beta). Math of the layer's own path, gdn.py:191-194:
 *   g = -exp(A_log[h]) * softplus(a + dt_bias[h]) (fp32; softplus(x) = x above 20),  beta = sigmoid(b).
 * a, b [n_tokens, HV] (any act dtype), A_log, dt_bias [HV] (param_dtype; dt_bias may be NULL), HV <= 1024.
 * Replaces: fla gdn_gate_chunk_cumsum / gdn_gate_bwd (fla/ops/gated_delta_rule/gate.py) and the in-kernel
 * beta sigmoid of FLA 0.5.2. gdn_gate_bwd writes da (dtype of a) and dA_log, ddt_bias (fp32 [HV], zeroed
 * by the call itself; ddt_bias is required iff dt_bias is given).
 */
int gdn_gate_fwd(int64_t n_tokens, int64_t HV, const void* a, int32_t a_dtype, const void* A_log,
                 const void* dt_bias, int32_t param_dtype, float* g_out, gdn_stream_t stream);
int gdn_gate_bwd(int64_t n_tokens, int64_t HV, const void* a, int32_t a_dtype, const void* A_log,
                 const void* dt_bias, int32_t param_dtype, const float* dg, void* da, float* dA_log,
                 float* ddt_bias, gdn_stream_t stream);
int gdn_beta_sigmoid_fwd(int64_t n, const void* b, int32_t b_dtype, float* beta_out, gdn_stream_t stream);
int gdn_beta_sigmoid_bwd(int64_t n, const void* b, int32_t b_dtype, const float* dbeta, void* db,
                         gdn_stream_t stream);

/*
 * The layer's output step in one pass: y = RMSNorm(x) * weight * silu(gate) per row of D features
 * (sore/model/gdn.py:180-188 with FLA's rms_norm_gated, activation "swish", no bias; RMSNorm of
 * sore/model/layers.py:15-18: x * rsqrt(mean(x^2) + eps), fp32 math, one rounding to the act dtype).
 * x, gate, y, dy, dx, dgate [rows, D] (act dtype), weight [D] (w_dtype), D a multiple of 32, <= 1024.
 * Replaces: fla.modules.fused_norm_gate.rms_norm_gated. The backward writes dx, dgate (act dtype) and
 * dweight (fp32 [D], zeroed by the call itself).
 */
int gdn_rms_norm_gated_fwd(int64_t rows, int64_t D, const void* x, const void* gate, int32_t act_dtype,
                           const void* weight, int32_t w_dtype, float eps, void* y, gdn_stream_t stream);
int gdn_rms_norm_gated_bwd(int64_t rows, int64_t D, const void* x, const void* gate, int32_t act_dtype,
                           const void* weight, int32_t w_dtype, float eps, const void* dy, void* dx,
                           void* dgate, float* dweight, gdn_stream_t stream);

/*
 * The layer's q/k/v prologue: short causal depthwise convolution, optionally followed by SiLU
 * (sore/model/conv.py:6-23, FLA causal_conv1d at sore/model/gdn.py:199-207):
 *   z[t, c] = sum_{j < K} w[c, K-1-j] x[t-j, c] over taps inside t's document,  y = silu(z) if silu.
 * x, y, dy, dx [B, T, C] (act dtype, 16-byte aligned, C a multiple of 8), weight [C, K] (w_dtype),
 * 1 <= K <= 4, C * K <= 16384. Documents are the batch rows, or with cu_seqlens (int64 [N+1], B == 1)
 * the packed spans. Replaces: fla.modules.conv.causal_conv1d (activation "silu", no bias, no cache).
 * The backward writes dx and dweight (fp32 [C, K], zeroed by the call itself).
 */
int gdn_causal_conv1d_fwd(int64_t B, int64_t T, int64_t C, int64_t K, const void* x, int32_t act_dtype,
                          const void* weight, int32_t w_dtype, const int64_t* cu_seqlens, int64_t N,
                          int32_t silu, void* y, gdn_stream_t stream);
int gdn_causal_conv1d_bwd(int64_t B, int64_t T, int64_t C, int64_t K, const void* x, int32_t act_dtype,
                          const void* weight, int32_t w_dtype, const int64_t* cu_seqlens, int64_t N,
                          int32_t silu, const void* dy, void* dx, float* dweight, gdn_stream_t stream);

/*
 * Sequence split (no counterpart in the reference, which has no context parallelism: soreRNN only
 * grows the context by curriculum, configs/b0_8_pretrain.yaml:18-20). A segment of tokens maps the
 * state entering it to S_out = M S_in + C, where C is gdn_chunk_fwd's final_state from a zero state
 * and M = prod_t exp(g_t)(I - beta_t k_t k_t^T) (later tokens on the left).
 *
 * gdn_segment_transition writes M as fp32 [N, HV, DK, DK]: it is the final state of the same
 * recurrence run with v = 0 from the identity state.
 */
int gdn_segment_transition(const gdn_problem* p, const void* k, const void* g, const void* beta,
                           float* transition, void* workspace, size_t workspace_bytes, gdn_stream_t stream);

/*
 * gdn_segment_apply_state adds the effect of an incoming state S_in [N, HV, DK, DV] to the outputs o of a
 * segment computed from a zero state:  o_t += scale (M_{<=t} S_in)^T q_t, which is the recurrence run
 * with v = 0 from S_in (the rule is linear in (S, v)). If final_state is not NULL it receives
 * final_state += M S_in, so that it becomes the segment's true outgoing state.
 */
int gdn_segment_apply_state(const gdn_problem* p, const void* q, const void* k, const void* g,
                            const void* beta, const float* state_in, void* o, float* final_state,
                            void* workspace, size_t workspace_bytes, gdn_stream_t stream);

/* Workspace bytes for the two sequence-split calls (same for both). */
size_t gdn_segment_workspace_size(const gdn_problem* p);

/*
 * The same sequence split on the chunked kernels (problems with gdn_uses_chunk_kernels(p) == 1; others get
 * GDN_ERR_SHAPE and use the two calls above). The chunk-parallel prep work of every (chunk, head) runs once
 * into `records` (gdn_segment_records_size(p) bytes, 16-byte aligned, kept by the caller between the calls),
 * and the per-sequence state passes reuse it:
 *   gdn_segment_maps    C = final_state of each sequence from initial_state (NULL = zeros), and, when
 *                       transition != NULL (needs DK == DV), M = the transition map [N, HV, DK, DK];
 *                       no outputs;
 *   gdn_segment_outputs o (and final_state, NULL = not wanted) of each sequence started from
 *                       incoming_state (NULL = zeros): the segment's true outputs once the caller has
 *                       composed its incoming state from the other segments' maps.
 * Three state passes in all, over one prep pass.
 * Replaces: the per-segment forward, gdn_segment_transition and gdn_segment_apply_state above.
 */
size_t gdn_segment_records_size(const gdn_problem* p);
int gdn_segment_maps(const gdn_problem* p, const void* q, const void* k, const void* v, const void* g,
                     const void* beta, const float* initial_state, float* final_state, float* transition,
                     void* records, size_t records_bytes, gdn_stream_t stream);
int gdn_segment_outputs(const gdn_problem* p, const void* q, const void* k, const void* v, const void* g,
                        const void* beta, const float* incoming_state, void* o, float* final_state, void* records,
                        size_t records_bytes, gdn_stream_t stream);

/*
 * The two calls above for training on pieces: each also writes its share of the backward's per-(chunk, head)
 * records into `saved` (gdn_chunk_saved_bytes(p) bytes, 16-byte aligned, the same buffer for both calls):
 * gdn_segment_maps_save the -W and T parts (prep pass), gdn_segment_outputs_save the S0^T, Delta^T and
 * Dd^T low parts from each sequence's true incoming state. After both, `saved` is what gdn_chunk_fwd_save
 * writes for the same problem started from those incoming states, so gdn_chunk_bwd_saved runs the reverse
 * sweep of any piece from a given end-state gradient (dht). This lets a caller cut long sequences into
 * pieces that run side by side when there are too few (sequence, head) pairs to fill the GPU.
 * Replaces: the same forward as gdn_chunk_fwd_save (fla chunk.py:365-380), split across pieces.
 */
int gdn_segment_maps_save(const gdn_problem* p, const void* q, const void* k, const void* v, const void* g,
                          const void* beta, const float* initial_state, float* final_state, float* transition,
                          void* saved, void* records, size_t records_bytes, gdn_stream_t stream);
int gdn_segment_outputs_save(const gdn_problem* p, const void* q, const void* k, const void* v, const void* g,
                             const void* beta, const float* incoming_state, void* o, float* final_state, void* saved,
                             void* records, size_t records_bytes, gdn_stream_t stream);

/*
 * The chain of piece maps along each of n_seq sequences cut into `pieces` pieces (training on pieces, with
 * gdn_segment_maps_save / gdn_segment_outputs_save / gdn_chunk_bwd_saved on the pieces as sequences). maps
 * [n_seq * pieces, HV, DK, DK] and terms, out [n_seq * pieces, HV, DK, DV] are fp32 with piece p of
 * sequence n at index n * pieces + p; start and final_state [n_seq, HV, DK, DV] (NULL = zeros / not wanted).
 *   reverse = 0: out[p] = the state entering piece p, given each piece's map (M_p, C_p = terms[p], the
 *                piece's final state from its own start, piece 0 from `start`): out[0] = start,
 *                out[p] = M_{p-1} out[p-1] + C_{p-1} for p >= 1 (as a chain: Y = C_0, Y <- M_p Y + C_p);
 *                final_state = the state leaving the last piece.
 *   reverse = 1: out[p] = the gradient of the state leaving piece p, given R_p = terms[p], the gradient
 *                entering piece p for a zero end-state gradient: out[pieces-1] = start (the gradient of
 *                the sequence's final state), out[p] = M_{p+1}^T out[p+1] + R_{p+1}.
 *   reverse = 2: as 0 with every term but terms[0] taken as zero; with terms = maps, final_state (required)
 *                = M_{pieces-1} ... M_1 M_0, the sequence's composite map; out (NULL = not wanted) = the
 *                prefix products M_{p-1} ... M_0 for p >= 1.
 * DK = DV = 128. fp32 throughout. No counterpart in the reference (it has no sequence split).
 */
int gdn_piece_chain(int64_t n_seq, int64_t pieces, int64_t HV, int64_t DK, int64_t DV, const float* maps,
                    const float* terms, const float* start, float* out, float* final_state, int32_t reverse,
                    gdn_stream_t stream);

/* Reads the error word that device-side bounded waits leave in `workspace` (0 = none; the word is
 * cleared at the start of every call that takes the workspace). Synchronises `stream`. */
int gdn_workspace_error(const void* workspace, gdn_stream_t stream, int32_t* error_out);

/* Reads and clears the device error words of the workspace-less streaming kernels (gdn_decode_step,
 * the norm-gate and conv entry points) on the current device: 0 = none, else the code of the first
 * kernel family whose bounded stage wait gave up (31 decode, 32 norm-gate, 33 conv). A kernel that gave
 * up stores nothing from then on (the decode step leaves those states unchanged). Synchronises `stream`.
 * No counterpart in the reference. */
int gdn_stream_kernels_error(gdn_stream_t stream, int32_t* error_out);

/* Number of kernels this library has launched in the process so far (host-side counter, for
 * benchmark accounting). No counterpart in the reference. */
uint64_t gdn_kernel_launches(void);

#ifdef __cplusplus
}
#endif
#endif /* GDN_B200_H */
