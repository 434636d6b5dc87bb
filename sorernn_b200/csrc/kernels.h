// Internal launch interfaces between the C ABI (gdn_abi.cu) and the kernel files.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/gdn_b200.h"

namespace gdn {

// Host-side count of kernel launches made by the library (gdn_kernel_launches()).
void count_launch(int n = 1);

// Validation of a gdn_problem (status code; GDN_OK when the problem is well formed).
int problem_status(const gdn_problem* p);

// Arguments of the recurrent (token-by-token) kernels.
struct RecLaunch {
    const void *q, *k, *v, *g, *beta;
    void* o;
    const float* h0;
    float* ht;
    const int64_t* cu;
    int64_t N, T, H, HV, DK, DV;
    float scale;
    int act_dtype, g_dtype, beta_dtype;
    int l2norm, zero_v, o_mode, h0_identity, ht_accumulate;
};

// Arguments of the chunked tcgen05 kernels (bf16 activations, DK = DV = 128).
struct ChunkLaunch {
    const void *q, *k, *v, *g, *beta;
    void* o;
    const float* h0;
    float* ht;
    float* ckpt;
    const int64_t* cu;
    int* err;  // device error word (bounded waits)
    int64_t B, T, N, H, HV;
    float scale;
    int g_dtype, beta_dtype, l2norm, zero_v, o_mode, h0_identity, ht_accumulate, ckpt_every;
    // recompute mode (used by the backward): when s0_out is set, ckpt is READ (the forward's checkpoints),
    // one CTA per (sequence, head, segment of ckpt_every chunks) restarts from its checkpoint and writes one
    // kBwdRecordBytes record per (chunk, head) to s0_out (the operand tiles listed below); no outputs, no
    // final state.
    void* s0_out;
    int64_t max_seqlen;
    // split forward only: when set, the prep and state passes also write the backward's kBwdRecordBytes record
    // of every (chunk, head) here (chunk_saved_bytes), so that the backward skips its recompute pass
    void* bwd_rec;
};

// Per-(chunk, head) record the backward sweep reads, written by the recompute pass or, in the saved-record
// mode, by the split forward (prep pass: -W, T; state pass: S0^T, Delta^T, Dd^T low): shared-memory images, in the
// 128-byte-swizzled operand layouts, of the chunk's S0^T (bf16 [dv][dk], 32 KB), -W (bf16 [j][dk], 16 KB),
// T = (I + A)^-1 (bf16 [i][j], 8 KB), Delta^T (bf16 [dv][j], 16 KB) and the low part of
// Dd^T = Delta^T diag(e^(G_C - G) / nk) relative to bf16(bf16(Delta^T) diag(...)) (16 KB).
constexpr size_t kBwdRecordBytes = 90112;
constexpr size_t kBwdRecW = 32768;    // -W then T: 24 KB contiguous
constexpr size_t kBwdRecT = 49152;
constexpr size_t kBwdRecDel = 57344;  // Delta^T
constexpr size_t kBwdRecDdl = 73728;  // Dd^T low part

// Per-(chunk, head) record of the split forward (gdn_chunk_split.cu): the prep pass writes it, the state
// pass reads it. Shared-memory images in the 128-byte-swizzled operand layouts of Qg = diag(scale e^G) Q
// (bf16 [i][dk], two 8 KB d-blocks), -W (bf16 [i][dk], two 8 KB d-blocks), TV = T diag(beta) (bf16 [i][j]),
// P hi and P lo (bf16 [i][j]), then fp32 vectors: e^(G_C - G_j) nk_j [64], nq_i [64], e^G_C.
constexpr size_t kFwdRecordBytes = 58368;
constexpr size_t kFwdRecQg = 0;
constexpr size_t kFwdRecW = 16384;
constexpr size_t kFwdRecTV = 32768;
constexpr size_t kFwdRecP = 40960;  // P hi, then P lo at +8192
constexpr size_t kFwdRecVec = 57344;
constexpr uint32_t kFwdRecVecBytes = 528;

// Arguments of the chunked backward.
struct ChunkBwdLaunch {
    const void *q, *k, *v, *g, *beta, *dout;
    const float *h0, *ckpt, *dht;
    void *dq, *dk, *dv;
    float *dg, *dbeta, *dh0;
    void* ws;  // chunk_bwd_workspace bytes
    const int64_t* cu;
    int* err;
    int64_t B, T, N, H, HV, max_seqlen;
    float scale;
    int g_dtype, beta_dtype, l2norm, ckpt_every;
    // records the split forward saved (chunk_saved_bytes); NULL: rebuild them from ckpt in a recompute pass
    const void* saved_rec;
    // 1: the sweep carries dS alone (no token gradients; dq .. dbeta unused) and writes dh0
    int state_grad_only;
};

// Codes the workspace-less streaming kernels leave in their device error words when a stage wait gives up
// (read through gdn_stream_kernels_error).
constexpr int GDN_DEV_ERR_DECODE = 31;
constexpr int GDN_DEV_ERR_NORM_GATE = 32;
constexpr int GDN_DEV_ERR_CONV = 33;
int read_clear_decode_error(cudaStream_t s, int* out);
int read_clear_norm_gate_error(cudaStream_t s, int* out);
int read_clear_conv_error(cudaStream_t s, int* out);

// Single-token decode for DK = DV = 128 (persistent bulk-copy pipeline over the fp32 states).
bool decode_tma_supported(int64_t DK, int64_t DV, const void* q, const void* k, const void* v, const float* state);
int decode_tma(const void* q, const void* k, const void* v, const void* g, const void* beta, float* state, void* o,
               int64_t N, int64_t H, int64_t HV, float scale, int act_dtype, int g_dtype, int beta_dtype, int l2norm,
               cudaStream_t s);

bool chunk_fwd_supported(int64_t DK, int64_t DV, int act_dtype);
int chunk_fwd(const ChunkLaunch& L, cudaStream_t s);
// The plain forward as two launches (chunk-parallel prep, per-(sequence, head) state pass); `ws` holds the
// per-chunk records (chunk_fwd_split_workspace bytes, 256-byte aligned).
size_t chunk_fwd_split_workspace(int64_t B, int64_t T, int64_t N, int64_t HV, bool varlen);
int chunk_fwd_split(const ChunkLaunch& L, void* ws, cudaStream_t s);
// The two launches of chunk_fwd_split on their own, over the same workspace: the prep pass writes the records
// (and, with cu_seqlens, each sequence's first chunk); the state pass reads them and may run several times
// (the sequence-split passes). The state pass honours zero_v, h0_identity and o == NULL (no outputs).
int chunk_prep_pass(const ChunkLaunch& L, void* ws, cudaStream_t s);
int chunk_state_pass(const ChunkLaunch& L, void* ws, cudaStream_t s);
bool chunk_bwd_supported(int64_t DK, int64_t DV, int act_dtype);
// workspace of chunk_bwd: the records (unless saved by the forward) and the fp32 dq/dk accumulators (HV > H)
size_t chunk_bwd_workspace(int64_t B, int64_t T, int64_t N, int64_t H, int64_t HV, bool varlen, bool saved);
// bytes of the backward records of every (chunk, head), as the split forward saves them
size_t chunk_saved_bytes(int64_t B, int64_t T, int64_t N, int64_t HV, bool varlen);
int chunk_bwd(const ChunkBwdLaunch& L, cudaStream_t s);

// The chain of piece maps along each sequence (gdn_piece_chain): mode 0 the states entering the pieces, mode 1
// the gradients of the pieces' end states, mode 2 the composite map (dk = dv = 128).
int piece_chain(int64_t n_seq, int64_t pieces, int64_t HV, const float* maps, const float* terms, const float* start,
                float* out, float* final_state, int mode, cudaStream_t s);

int rec_fwd(const RecLaunch& L, cudaStream_t s);
size_t rec_bwd_workspace(int64_t N, int64_t HV, int64_t DK, int64_t DV, int64_t max_len, int64_t total_tokens,
                         int64_t H);
int rec_bwd(const RecLaunch& L, const void* dout, const float* dht, void* dq, void* dk, void* dv, float* dg,
            float* dbeta, float* dh0, void* ws, int64_t max_len, int64_t total_tokens, cudaStream_t s);

}  // namespace gdn
