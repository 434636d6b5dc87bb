// extern "C" entry points declared in include/gdn_b200.h: host-side validation and dispatch.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

#include <atomic>

using namespace gdn;

namespace gdn {
static std::atomic<uint64_t> g_launches{0};
void count_launch(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }
}  // namespace gdn

namespace {

constexpr int64_t kChunk = 64;
constexpr size_t kErrBytes = 256;  // head of every workspace: device error word (bounded waits)

bool dtype_ok(int32_t d) { return d == GDN_BF16 || d == GDN_FP16 || d == GDN_FP32; }

int check_problem(const gdn_problem* p) {
    if (!p) return GDN_ERR_ARGUMENT;
    if (p->B < 0 || p->T < 0 || p->H <= 0 || p->HV <= 0 || p->DK <= 0 || p->DV <= 0 || p->N < 0) return GDN_ERR_SHAPE;
    if (p->HV % p->H) return GDN_ERR_SHAPE;
    if (p->DK > 128 || p->DV > 128) return GDN_ERR_SHAPE;
    if (p->cu_seqlens) {
        if (p->B != 1) return GDN_ERR_SHAPE;  // gdn_ref.py:42-43
    } else if (p->N != p->B) {
        return GDN_ERR_SHAPE;
    }
    if (!dtype_ok(p->act_dtype) || !dtype_ok(p->g_dtype) || !dtype_ok(p->beta_dtype)) return GDN_ERR_DTYPE;
    if (p->ckpt_every < 1) return GDN_ERR_ARGUMENT;
    return GDN_OK;
}

int64_t max_len(const gdn_problem* p) {
    if (p->max_seqlen > 0) return p->max_seqlen;
    return p->cu_seqlens ? p->B * p->T : p->T;
}

RecLaunch rec_launch(const gdn_problem* p) {
    RecLaunch L{};
    L.cu = p->cu_seqlens;
    L.N = p->N;
    L.T = p->T;
    L.H = p->H;
    L.HV = p->HV;
    L.DK = p->DK;
    L.DV = p->DV;
    L.scale = p->scale;
    L.act_dtype = p->act_dtype;
    L.g_dtype = p->g_dtype;
    L.beta_dtype = p->beta_dtype;
    L.l2norm = p->use_qk_l2norm;
    return L;
}

bool aligned16(const void* x) { return ((uintptr_t)x & 15) == 0; }

}  // namespace

namespace gdn {
int problem_status(const gdn_problem* p) { return check_problem(p); }
}  // namespace gdn

extern "C" {

const char* gdn_status_string(int status) {
    switch (status) {
        case GDN_OK: return "ok";
        case GDN_ERR_SHAPE: return "unsupported or inconsistent shape";
        case GDN_ERR_DTYPE: return "unsupported dtype";
        case GDN_ERR_ALIGN: return "pointer not 16-byte aligned";
        case GDN_ERR_LAUNCH: return "CUDA launch failed";
        case GDN_ERR_TIMEOUT: return "device-side wait timed out";
        case GDN_ERR_WORKSPACE: return "workspace missing or too small";
        case GDN_ERR_ARGUMENT: return "invalid argument";
        case GDN_ERR_SCRATCH_LIMIT: return "problem exceeds the no-allocation scratch limit (36 MiB)";
        default: return "unknown status";
    }
}

int gdn_uses_chunk_kernels(const gdn_problem* p) {
    return check_problem(p) == GDN_OK && chunk_fwd_supported(p->DK, p->DV, p->act_dtype) ? 1 : 0;
}

// Forward-type pass (plain forward, transition map, incoming-state correction): the chunked tcgen05
// kernel when the problem fits it, else the recurrent kernel.
static int dispatch_forward(const gdn_problem* p, const RecLaunch& L, float* ckpt, void* workspace, cudaStream_t s) {
    if (!gdn_uses_chunk_kernels(p)) return rec_fwd(L, s);
    ChunkLaunch C{};
    C.q = L.q; C.k = L.k; C.v = L.v; C.g = L.g; C.beta = L.beta; C.o = L.o;
    C.h0 = L.h0; C.ht = L.ht; C.ckpt = ckpt; C.cu = L.cu; C.err = (int*)workspace;
    C.B = p->B; C.T = p->T; C.N = p->N; C.H = p->H; C.HV = p->HV;
    C.scale = L.scale; C.g_dtype = L.g_dtype; C.beta_dtype = L.beta_dtype; C.l2norm = L.l2norm;
    C.zero_v = L.zero_v; C.o_mode = L.o_mode; C.h0_identity = L.h0_identity; C.ht_accumulate = L.ht_accumulate;
    C.ckpt_every = p->ckpt_every;
    return chunk_fwd(C, s);
}

int64_t gdn_checkpoint_count(const gdn_problem* p) {
    if (check_problem(p) != GDN_OK) return -1;
    const int64_t K = p->ckpt_every;
    if (!p->cu_seqlens) {
        const int64_t nc = (p->T + kChunk - 1) / kChunk;
        return p->N * ((nc + K - 1) / K);
    }
    // sum_n ceil(ceil(len_n / 64) / K) <= (sum_n ceil(len_n / 64)) / K + N <= (T + 63 N) / 64 / K + N
    const int64_t nc = (p->B * p->T + (kChunk - 1) * p->N) / kChunk;
    return nc / K + p->N + 1;
}

size_t gdn_chunk_fwd_workspace_size(const gdn_problem* p) {
    if (check_problem(p) != GDN_OK) return 0;
    if (!gdn_uses_chunk_kernels(p)) return kErrBytes;
    return kErrBytes + chunk_fwd_split_workspace(p->B, p->T, p->N, p->HV, p->cu_seqlens != nullptr);
}

size_t gdn_chunk_bwd_workspace_size(const gdn_problem* p) {
    if (check_problem(p) != GDN_OK) return 0;
    if (gdn_uses_chunk_kernels(p))
        return kErrBytes + chunk_bwd_workspace(p->B, p->T, p->N, p->H, p->HV, p->cu_seqlens, false);
    return kErrBytes + rec_bwd_workspace(p->N, p->HV, p->DK, p->DV, max_len(p), p->B * p->T, p->H);
}

size_t gdn_chunk_saved_bytes(const gdn_problem* p) {
    if (!gdn_uses_chunk_kernels(p)) return 0;
    return chunk_saved_bytes(p->B, p->T, p->N, p->HV, p->cu_seqlens != nullptr);
}

size_t gdn_chunk_bwd_saved_workspace_size(const gdn_problem* p) {
    if (!gdn_uses_chunk_kernels(p)) return 0;
    return kErrBytes + chunk_bwd_workspace(p->B, p->T, p->N, p->H, p->HV, p->cu_seqlens, true);
}

// gdn_chunk_fwd (checkpoints) and gdn_chunk_fwd_save (saved: the backward's per-chunk records)
static int forward_impl(const gdn_problem* p, const void* q, const void* k, const void* v, const void* g,
                        const void* beta, const float* initial_state, void* o, float* final_state,
                        float* checkpoints, void* saved, void* workspace, size_t workspace_bytes,
                        gdn_stream_t stream) {
    int st = check_problem(p);
    if (st != GDN_OK) return st;
    cudaStream_t s = (cudaStream_t)stream;
    if (p->B * p->T == 0) {  // no tokens: the final state is the initial state (token pointers may be null)
        if (!final_state) return GDN_OK;
        const size_t bytes = (size_t)p->N * p->HV * p->DK * p->DV * sizeof(float);
        if (bytes == 0) return GDN_OK;
        const cudaError_t e = initial_state ? cudaMemcpyAsync(final_state, initial_state, bytes,
                                                              cudaMemcpyDeviceToDevice, s)
                                            : cudaMemsetAsync(final_state, 0, bytes, s);
        return e == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
    }
    if (!q || !k || !v || !g || !beta || !o) return GDN_ERR_ARGUMENT;
    if (!workspace || workspace_bytes < gdn_chunk_fwd_workspace_size(p)) return GDN_ERR_WORKSPACE;
    if (cudaMemsetAsync(workspace, 0, kErrBytes, s) != cudaSuccess) return GDN_ERR_LAUNCH;
    RecLaunch L = rec_launch(p);
    L.q = q; L.k = k; L.v = v; L.g = g; L.beta = beta; L.o = o;
    L.h0 = initial_state;
    L.ht = final_state;
    if (gdn_uses_chunk_kernels(p)) {  // chunk-parallel prep + per-(sequence, head) state pass
        ChunkLaunch C{};
        C.q = q; C.k = k; C.v = v; C.g = g; C.beta = beta; C.o = o;
        C.h0 = initial_state; C.ht = final_state; C.ckpt = checkpoints; C.cu = p->cu_seqlens;
        C.err = (int*)workspace;
        C.B = p->B; C.T = p->T; C.N = p->N; C.H = p->H; C.HV = p->HV; C.max_seqlen = max_len(p);
        C.scale = p->scale; C.g_dtype = p->g_dtype; C.beta_dtype = p->beta_dtype; C.l2norm = p->use_qk_l2norm;
        C.ckpt_every = p->ckpt_every;
        C.bwd_rec = saved;
        return chunk_fwd_split(C, (char*)workspace + kErrBytes, s);
    }
    return dispatch_forward(p, L, checkpoints, workspace, s);
}

int gdn_chunk_fwd(const gdn_problem* p, const void* q, const void* k, const void* v, const void* g,
                  const void* beta, const float* initial_state, void* o, float* final_state, float* checkpoints,
                  void* workspace, size_t workspace_bytes, gdn_stream_t stream) {
    return forward_impl(p, q, k, v, g, beta, initial_state, o, final_state, checkpoints, nullptr, workspace,
                        workspace_bytes, stream);
}

int gdn_chunk_fwd_save(const gdn_problem* p, const void* q, const void* k, const void* v, const void* g,
                       const void* beta, const float* initial_state, void* o, float* final_state, void* saved,
                       void* workspace, size_t workspace_bytes, gdn_stream_t stream) {
    int st = check_problem(p);
    if (st != GDN_OK) return st;
    if (!gdn_uses_chunk_kernels(p)) return GDN_ERR_SHAPE;
    if (p->B * p->T > 0 && !saved) return GDN_ERR_ARGUMENT;
    if (saved && !aligned16(saved)) return GDN_ERR_ALIGN;
    return forward_impl(p, q, k, v, g, beta, initial_state, o, final_state, nullptr, saved, workspace,
                        workspace_bytes, stream);
}

// gdn_chunk_bwd (from checkpoints) and gdn_chunk_bwd_saved (from the records gdn_chunk_fwd_save wrote)
static int backward_impl(const gdn_problem* p, const void* q, const void* k, const void* v, const void* g,
                         const void* beta, const float* initial_state, const float* checkpoints, const void* saved,
                         const void* dout, const float* dht, void* dq, void* dk, void* dv, float* dg,
                         float* dbeta, float* dh0, void* workspace, size_t workspace_bytes, size_t workspace_need,
                         gdn_stream_t stream) {
    int st = check_problem(p);
    if (st != GDN_OK) return st;
    cudaStream_t s = (cudaStream_t)stream;
    if (p->B * p->T == 0) {  // no tokens: dh0 is dht (token pointers may be null)
        if (!dh0) return GDN_OK;
        const size_t bytes = (size_t)p->N * p->HV * p->DK * p->DV * sizeof(float);
        if (bytes == 0) return GDN_OK;
        const cudaError_t e = dht ? cudaMemcpyAsync(dh0, dht, bytes, cudaMemcpyDeviceToDevice, s)
                                  : cudaMemsetAsync(dh0, 0, bytes, s);
        return e == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
    }
    if (!q || !k || !v || !g || !beta || !dout || !dq || !dk || !dv || !dg || !dbeta) return GDN_ERR_ARGUMENT;
    if (!workspace || workspace_bytes < workspace_need) return GDN_ERR_WORKSPACE;
    if (!aligned16(workspace)) return GDN_ERR_ALIGN;
    if (cudaMemsetAsync(workspace, 0, kErrBytes, s) != cudaSuccess) return GDN_ERR_LAUNCH;
    if (gdn_uses_chunk_kernels(p)) {
        // the chunked backward reads the forward's saved records, or restarts from its checkpoints
        if (!checkpoints && !saved) return GDN_ERR_ARGUMENT;
        ChunkBwdLaunch C{};
        C.q = q; C.k = k; C.v = v; C.g = g; C.beta = beta; C.dout = dout;
        C.h0 = initial_state; C.ckpt = checkpoints; C.dht = dht;
        C.dq = dq; C.dk = dk; C.dv = dv; C.dg = dg; C.dbeta = dbeta; C.dh0 = dh0;
        C.ws = (char*)workspace + kErrBytes; C.cu = p->cu_seqlens; C.err = (int*)workspace;
        C.B = p->B; C.T = p->T; C.N = p->N; C.H = p->H; C.HV = p->HV; C.max_seqlen = max_len(p);
        C.scale = p->scale; C.g_dtype = p->g_dtype; C.beta_dtype = p->beta_dtype; C.l2norm = p->use_qk_l2norm;
        C.ckpt_every = p->ckpt_every;
        C.saved_rec = saved;
        return chunk_bwd(C, s);
    }
    RecLaunch L = rec_launch(p);
    L.q = q; L.k = k; L.v = v; L.g = g; L.beta = beta;
    L.h0 = initial_state;
    return rec_bwd(L, dout, dht, dq, dk, dv, dg, dbeta, dh0, (char*)workspace + kErrBytes, max_len(p),
                   p->B * p->T, s);
}

int gdn_chunk_bwd(const gdn_problem* p, const void* q, const void* k, const void* v, const void* g,
                  const void* beta, const float* initial_state, const float* checkpoints, const void* dout,
                  const float* dht, void* dq, void* dk, void* dv, float* dg, float* dbeta, float* dh0,
                  void* workspace, size_t workspace_bytes, gdn_stream_t stream) {
    return backward_impl(p, q, k, v, g, beta, initial_state, checkpoints, nullptr, dout, dht, dq, dk, dv, dg, dbeta,
                         dh0, workspace, workspace_bytes, gdn_chunk_bwd_workspace_size(p), stream);
}

int gdn_chunk_bwd_saved(const gdn_problem* p, const void* q, const void* k, const void* v, const void* g,
                        const void* beta, const void* saved, const void* dout, const float* dht, void* dq, void* dk,
                        void* dv, float* dg, float* dbeta, float* dh0, void* workspace, size_t workspace_bytes,
                        gdn_stream_t stream) {
    int st = check_problem(p);
    if (st != GDN_OK) return st;
    if (!gdn_uses_chunk_kernels(p)) return GDN_ERR_SHAPE;
    if (p->B * p->T > 0 && !saved) return GDN_ERR_ARGUMENT;
    if (saved && !aligned16(saved)) return GDN_ERR_ALIGN;
    return backward_impl(p, q, k, v, g, beta, nullptr, nullptr, saved, dout, dht, dq, dk, dv, dg, dbeta, dh0,
                         workspace, workspace_bytes, gdn_chunk_bwd_saved_workspace_size(p), stream);
}

int gdn_chunk_state_grad_saved(const gdn_problem* p, const void* q, const void* k, const void* v, const void* g,
                               const void* beta, const void* saved, const void* dout, const float* dht, float* dh0,
                               void* workspace, size_t workspace_bytes, gdn_stream_t stream) {
    int st = check_problem(p);
    if (st != GDN_OK) return st;
    if (!gdn_uses_chunk_kernels(p)) return GDN_ERR_SHAPE;
    if (!dh0) return GDN_ERR_ARGUMENT;
    cudaStream_t s = (cudaStream_t)stream;
    if (p->B * p->T == 0) {  // no tokens: dh0 is dht
        const size_t bytes = (size_t)p->N * p->HV * p->DK * p->DV * sizeof(float);
        if (bytes == 0) return GDN_OK;
        const cudaError_t e = dht ? cudaMemcpyAsync(dh0, dht, bytes, cudaMemcpyDeviceToDevice, s)
                                  : cudaMemsetAsync(dh0, 0, bytes, s);
        return e == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
    }
    if (!q || !k || !v || !g || !beta || !dout || !saved) return GDN_ERR_ARGUMENT;
    if (!aligned16(saved)) return GDN_ERR_ALIGN;
    if (!workspace || workspace_bytes < gdn_chunk_bwd_saved_workspace_size(p)) return GDN_ERR_WORKSPACE;
    if (!aligned16(workspace)) return GDN_ERR_ALIGN;
    if (cudaMemsetAsync(workspace, 0, kErrBytes, s) != cudaSuccess) return GDN_ERR_LAUNCH;
    ChunkBwdLaunch C{};
    C.q = q; C.k = k; C.v = v; C.g = g; C.beta = beta; C.dout = dout; C.dht = dht; C.dh0 = dh0;
    C.ws = (char*)workspace + kErrBytes; C.cu = p->cu_seqlens; C.err = (int*)workspace;
    C.B = p->B; C.T = p->T; C.N = p->N; C.H = p->H; C.HV = p->HV; C.max_seqlen = max_len(p);
    C.scale = p->scale; C.g_dtype = p->g_dtype; C.beta_dtype = p->beta_dtype; C.l2norm = p->use_qk_l2norm;
    C.ckpt_every = p->ckpt_every;
    C.saved_rec = saved;
    C.state_grad_only = 1;
    return chunk_bwd(C, s);
}

int gdn_decode_step(int64_t N, int64_t H, int64_t HV, int64_t DK, int64_t DV, float scale, int32_t act_dtype,
                    int32_t g_dtype, int32_t beta_dtype, int32_t use_qk_l2norm, const void* q, const void* k,
                    const void* v, const void* g, const void* beta, float* state, void* o, gdn_stream_t stream) {
    if (N < 0 || H <= 0 || HV <= 0 || HV % H || DK <= 0 || DV <= 0 || DK > 128 || DV > 128) return GDN_ERR_SHAPE;
    if (!dtype_ok(act_dtype) || !dtype_ok(g_dtype) || !dtype_ok(beta_dtype)) return GDN_ERR_DTYPE;
    if (!q || !k || !v || !g || !beta || !state || !o) return GDN_ERR_ARGUMENT;
    if (DV == 128 && !aligned16(state)) return GDN_ERR_ALIGN;
    if (decode_tma_supported(DK, DV, q, k, v, state))
        return decode_tma(q, k, v, g, beta, state, o, N, H, HV, scale, act_dtype, g_dtype, beta_dtype,
                          use_qk_l2norm, (cudaStream_t)stream);
    RecLaunch L{};
    L.q = q; L.k = k; L.v = v; L.g = g; L.beta = beta; L.o = o;
    L.h0 = state;
    L.ht = state;  // in place: every CTA reads its whole state into registers before writing it
    L.cu = nullptr;
    L.N = N; L.T = 1; L.H = H; L.HV = HV; L.DK = DK; L.DV = DV;
    L.scale = scale;
    L.act_dtype = act_dtype; L.g_dtype = g_dtype; L.beta_dtype = beta_dtype;
    L.l2norm = use_qk_l2norm;
    return rec_fwd(L, (cudaStream_t)stream);
}

size_t gdn_segment_workspace_size(const gdn_problem* p) {
    if (check_problem(p) != GDN_OK) return 0;
    return kErrBytes;
}

int gdn_segment_transition(const gdn_problem* p, const void* k, const void* g, const void* beta, float* transition,
                           void* workspace, size_t workspace_bytes, gdn_stream_t stream) {
    int st = check_problem(p);
    if (st != GDN_OK) return st;
    if (p->DK != p->DV) return GDN_ERR_SHAPE;  // the map is run as a DK x DK state
    if (!k || !g || !beta || !transition) return GDN_ERR_ARGUMENT;
    if (!workspace || workspace_bytes < gdn_segment_workspace_size(p)) return GDN_ERR_WORKSPACE;
    cudaStream_t s = (cudaStream_t)stream;
    if (cudaMemsetAsync(workspace, 0, kErrBytes, s) != cudaSuccess) return GDN_ERR_LAUNCH;
    RecLaunch L = rec_launch(p);
    L.q = k; L.k = k; L.v = k; L.g = g; L.beta = beta; L.o = nullptr;
    L.zero_v = 1;
    L.o_mode = 2;
    L.h0_identity = 1;
    L.ht = transition;
    return dispatch_forward(p, L, nullptr, workspace, s);
}

int gdn_segment_apply_state(const gdn_problem* p, const void* q, const void* k, const void* g, const void* beta,
                            const float* state_in, void* o, float* final_state, void* workspace,
                            size_t workspace_bytes, gdn_stream_t stream) {
    int st = check_problem(p);
    if (st != GDN_OK) return st;
    if (!q || !k || !g || !beta || !state_in || !o) return GDN_ERR_ARGUMENT;
    if (!workspace || workspace_bytes < gdn_segment_workspace_size(p)) return GDN_ERR_WORKSPACE;
    cudaStream_t s = (cudaStream_t)stream;
    if (cudaMemsetAsync(workspace, 0, kErrBytes, s) != cudaSuccess) return GDN_ERR_LAUNCH;
    RecLaunch L = rec_launch(p);
    L.q = q; L.k = k; L.v = q; L.g = g; L.beta = beta; L.o = o;
    L.zero_v = 1;
    L.o_mode = 1;
    L.h0 = state_in;
    L.ht = final_state;  // final_state += M S_in (may be NULL)
    L.ht_accumulate = 1;
    return dispatch_forward(p, L, nullptr, workspace, s);
}

// count matrices [D, D] set to the identity (the transition map of an empty segment)
__global__ void identity_states_kernel(float* m, int64_t count, int64_t D) {
    const int64_t n = count * D * D;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i % (D * D);
        m[i] = r / D == r % D ? 1.f : 0.f;
    }
}

size_t gdn_segment_records_size(const gdn_problem* p) {
    if (!gdn_uses_chunk_kernels(p)) return 0;
    return kErrBytes + chunk_fwd_split_workspace(p->B, p->T, p->N, p->HV, p->cu_seqlens != nullptr);
}

static ChunkLaunch segment_launch(const gdn_problem* p, const void* q, const void* k, const void* v, const void* g,
                                  const void* beta, void* records) {
    ChunkLaunch C{};
    C.q = q; C.k = k; C.v = v; C.g = g; C.beta = beta; C.cu = p->cu_seqlens;
    C.err = (int*)records;
    C.B = p->B; C.T = p->T; C.N = p->N; C.H = p->H; C.HV = p->HV; C.max_seqlen = max_len(p);
    C.scale = p->scale; C.g_dtype = p->g_dtype; C.beta_dtype = p->beta_dtype; C.l2norm = p->use_qk_l2norm;
    C.ckpt_every = p->ckpt_every;
    return C;
}

static int segment_maps_impl(const gdn_problem* p, const void* q, const void* k, const void* v, const void* g,
                             const void* beta, const float* initial_state, float* final_state, float* transition,
                             void* saved, void* records, size_t records_bytes, gdn_stream_t stream) {
    int st = check_problem(p);
    if (st != GDN_OK) return st;
    if (!gdn_uses_chunk_kernels(p)) return GDN_ERR_SHAPE;
    if (!q || !k || !v || !g || !beta || !final_state) return GDN_ERR_ARGUMENT;
    if (!records || records_bytes < gdn_segment_records_size(p)) return GDN_ERR_WORKSPACE;
    if (!aligned16(records) || (saved && !aligned16(saved))) return GDN_ERR_ALIGN;
    cudaStream_t s = (cudaStream_t)stream;
    if (cudaMemsetAsync(records, 0, kErrBytes, s) != cudaSuccess) return GDN_ERR_LAUNCH;
    if (p->B * p->T == 0) {  // no tokens: C is the initial state and M the identity
        const size_t bytes = (size_t)p->N * p->HV * p->DK * p->DV * sizeof(float);
        if (bytes == 0) return GDN_OK;
        const cudaError_t e = initial_state ? cudaMemcpyAsync(final_state, initial_state, bytes,
                                                              cudaMemcpyDeviceToDevice, s)
                                            : cudaMemsetAsync(final_state, 0, bytes, s);
        if (e != cudaSuccess) return GDN_ERR_LAUNCH;
        if (transition) {
            identity_states_kernel<<<148, 256, 0, s>>>(transition, p->N * p->HV, p->DK);
            count_launch();
            if (cudaGetLastError() != cudaSuccess) return GDN_ERR_LAUNCH;
        }
        return GDN_OK;
    }
    void* ws = (char*)records + kErrBytes;
    ChunkLaunch C = segment_launch(p, q, k, v, g, beta, records);
    C.bwd_rec = saved;  // the prep pass writes the records' -W and T parts; the state passes below write nothing
    if ((st = chunk_prep_pass(C, ws, s)) != GDN_OK) return st;
    C.bwd_rec = nullptr;
    C.h0 = initial_state;  // C: the final state from the initial state, no outputs
    C.ht = final_state;
    if ((st = chunk_state_pass(C, ws, s)) != GDN_OK) return st;
    if (!transition) return GDN_OK;
    C.h0 = nullptr;  // M: the state from the identity with v = 0
    C.h0_identity = 1;
    C.zero_v = 1;
    C.ht = transition;
    return chunk_state_pass(C, ws, s);
}

static int segment_outputs_impl(const gdn_problem* p, const void* q, const void* k, const void* v, const void* g,
                                const void* beta, const float* incoming_state, void* o, float* final_state,
                                void* saved, void* records, size_t records_bytes, gdn_stream_t stream) {
    int st = check_problem(p);
    if (st != GDN_OK) return st;
    if (!gdn_uses_chunk_kernels(p)) return GDN_ERR_SHAPE;
    if (p->B * p->T == 0) return GDN_OK;
    if (!q || !k || !v || !g || !beta || !o) return GDN_ERR_ARGUMENT;
    if (!records || records_bytes < gdn_segment_records_size(p)) return GDN_ERR_WORKSPACE;
    if (!aligned16(records) || (saved && !aligned16(saved))) return GDN_ERR_ALIGN;
    ChunkLaunch C = segment_launch(p, q, k, v, g, beta, records);
    C.o = o;
    C.h0 = incoming_state;
    C.ht = final_state;
    C.bwd_rec = saved;  // S0^T, Delta^T and the Dd^T low part of every chunk, from the true incoming state
    return chunk_state_pass(C, (char*)records + kErrBytes, (cudaStream_t)stream);
}

int gdn_segment_maps(const gdn_problem* p, const void* q, const void* k, const void* v, const void* g,
                     const void* beta, const float* initial_state, float* final_state, float* transition,
                     void* records, size_t records_bytes, gdn_stream_t stream) {
    return segment_maps_impl(p, q, k, v, g, beta, initial_state, final_state, transition, nullptr, records,
                             records_bytes, stream);
}

int gdn_segment_outputs(const gdn_problem* p, const void* q, const void* k, const void* v, const void* g,
                        const void* beta, const float* incoming_state, void* o, float* final_state, void* records,
                        size_t records_bytes, gdn_stream_t stream) {
    return segment_outputs_impl(p, q, k, v, g, beta, incoming_state, o, final_state, nullptr, records,
                                records_bytes, stream);
}

int gdn_segment_maps_save(const gdn_problem* p, const void* q, const void* k, const void* v, const void* g,
                          const void* beta, const float* initial_state, float* final_state, float* transition,
                          void* saved, void* records, size_t records_bytes, gdn_stream_t stream) {
    if (p && p->B * p->T > 0 && !saved) return GDN_ERR_ARGUMENT;
    return segment_maps_impl(p, q, k, v, g, beta, initial_state, final_state, transition, saved, records,
                             records_bytes, stream);
}

int gdn_segment_outputs_save(const gdn_problem* p, const void* q, const void* k, const void* v, const void* g,
                             const void* beta, const float* incoming_state, void* o, float* final_state, void* saved,
                             void* records, size_t records_bytes, gdn_stream_t stream) {
    if (p && p->B * p->T > 0 && !saved) return GDN_ERR_ARGUMENT;
    return segment_outputs_impl(p, q, k, v, g, beta, incoming_state, o, final_state, saved, records, records_bytes,
                                stream);
}

int gdn_piece_chain(int64_t n_seq, int64_t pieces, int64_t HV, int64_t DK, int64_t DV, const float* maps,
                    const float* terms, const float* start, float* out, float* final_state, int32_t reverse,
                    gdn_stream_t stream) {
    const int mode = reverse;  // 0 forward, 1 reverse, 2 composite map
    if (n_seq < 0 || pieces < 0 || HV < 0) return GDN_ERR_SHAPE;
    if (DK != 128 || DV != 128) return GDN_ERR_SHAPE;
    if (mode < 0 || mode > 2) return GDN_ERR_ARGUMENT;
    if (n_seq * pieces * HV == 0) return GDN_OK;
    if (!terms || (pieces > 1 && !maps)) return GDN_ERR_ARGUMENT;
    if (mode == 2 ? !final_state : !out) return GDN_ERR_ARGUMENT;
    if (!aligned16(maps) || !aligned16(terms) || !aligned16(out) || !aligned16(start) || !aligned16(final_state))
        return GDN_ERR_ALIGN;
    return piece_chain(n_seq, pieces, HV, maps, terms, start, out, final_state, mode, (cudaStream_t)stream);
}

uint64_t gdn_kernel_launches(void) { return g_launches.load(std::memory_order_relaxed); }

int gdn_stream_kernels_error(gdn_stream_t stream, int32_t* error_out) {
    if (!error_out) return GDN_ERR_ARGUMENT;
    cudaStream_t s = (cudaStream_t)stream;
    int e[3] = {0, 0, 0};
    if (read_clear_decode_error(s, &e[0]) != GDN_OK || read_clear_norm_gate_error(s, &e[1]) != GDN_OK ||
        read_clear_conv_error(s, &e[2]) != GDN_OK)
        return GDN_ERR_LAUNCH;
    if (cudaStreamSynchronize(s) != cudaSuccess) return GDN_ERR_LAUNCH;
    *error_out = e[0] ? e[0] : (e[1] ? e[1] : e[2]);
    return GDN_OK;
}

int gdn_workspace_error(const void* workspace, gdn_stream_t stream, int32_t* error_out) {
    if (!workspace || !error_out) return GDN_ERR_ARGUMENT;
    if (cudaMemcpyAsync(error_out, workspace, sizeof(int32_t), cudaMemcpyDeviceToHost, (cudaStream_t)stream) !=
        cudaSuccess)
        return GDN_ERR_LAUNCH;
    if (cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess) return GDN_ERR_LAUNCH;
    return GDN_OK;
}

}  // extern "C"
