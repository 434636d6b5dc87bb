// Recurrent (token-by-token) gated delta rule kernels: fp32 state in registers, fp32 arithmetic.
//
// These run the reference recurrence (soreRNN sore/model/gdn_ref.py:17-22) literally, one token at a
// time, so they match the fp32 oracle to rounding. They serve
//   * the single-token decode step (HBM-bound: one 128-bit vectorised read and write of the state),
//   * fp32 inputs (the reference-precision mode; tensor cores would be TF32/bf16),
//   * head sizes the chunked tcgen05 kernels do not cover (DK, DV <= 128).
//
// Thread layout: NW warps per (sequence, value head); warp w owns state rows i = w + NW r
// (r < RPT = 128 / NW); lane l owns columns 4l..4l+3 (VEC4, DV == 128: float4 accesses, each warp
// row access is one 512-byte coalesced segment) or l + 32c otherwise. Reductions over rows (S^T k,
// S^T q) go through shared memory across the warps; reductions over columns are warp shuffles.
#include "common.cuh"
#include "kernels.h"

namespace gdn {

struct RecFwdArgs {
    const void *q, *k, *v, *g, *beta;
    int g_dtype, beta_dtype;
    void* o;
    const float* h0;
    float* ht;
    const int64_t* cu;
    int64_t T;  // tokens per batch row when cu == nullptr
    int H, HV, DK, DV;
    float scale;
    int l2norm;
    int zero_v;         // treat v as zero (sequence-split passes)
    int o_mode;         // 0 write, 1 accumulate (o += ...), 2 skip
    int h0_identity;    // start from the identity (DK == DV) instead of h0/zeros
    int ht_accumulate;  // ht += final state instead of ht = final state
};

template <bool VEC4> __device__ __forceinline__ int col_of(int l, int c) { return VEC4 ? 4 * l + c : l + 32 * c; }

template <int NW> struct TokenSmem {
    float q[128], k[128], v[128], dout[128];
    float red[2][NW][128];
    float sc[8];  // gamma, beta, 1/|q|, 1/|k|, q.k (normalised), |q|, |k|, scratch
    float rowq[128], rowk[128];
    float part[NW][2];
};

__device__ __forceinline__ float ld_any(const void* p, int dtype, int64_t i) {
    if (dtype == GDN_FP32) return ((const float*)p)[i];
    if (dtype == GDN_BF16) return __bfloat162float(((const __nv_bfloat16*)p)[i]);
    return __half2float(((const __half*)p)[i]);
}

// Loads token t's q, k, v (and do), g, beta into smem and the norms (warp 0). Barrier on both sides.
template <int NW, typename TA>
__device__ __forceinline__ void load_token(TokenSmem<NW>& sm, const RecFwdArgs& a, int64_t t, int hq, int hv,
                                           const TA* dout) {
    const int tid = threadIdx.x;
    __syncthreads();
    if (tid < a.DK) {
        sm.q[tid] = ld((const TA*)a.q, (t * a.H + hq) * a.DK + tid);
        sm.k[tid] = ld((const TA*)a.k, (t * a.H + hq) * a.DK + tid);
    }
    if (tid < a.DV) {
        sm.v[tid] = a.zero_v ? 0.f : ld((const TA*)a.v, (t * a.HV + hv) * a.DV + tid);
        if (dout) sm.dout[tid] = ld(dout, (t * a.HV + hv) * a.DV + tid);
    }
    __syncthreads();
    if (tid < 32) {
        float nq = 0.f, nk = 0.f, qk = 0.f;
        for (int i = tid; i < a.DK; i += 32) {
            nq += sm.q[i] * sm.q[i];
            nk += sm.k[i] * sm.k[i];
            qk += sm.q[i] * sm.k[i];
        }
        nq = warp_sum(nq);
        nk = warp_sum(nk);
        qk = warp_sum(qk);
        if (tid == 0) {
            float iq = 1.f, ik = 1.f, lq = 1.f, lk = 1.f;
            if (a.l2norm) {
                lq = fmaxf(sqrtf(nq), kL2Eps);
                lk = fmaxf(sqrtf(nk), kL2Eps);
                iq = 1.f / lq;
                ik = 1.f / lk;
            }
            sm.sc[0] = __expf(ld_any(a.g, a.g_dtype, t * a.HV + hv));
            sm.sc[1] = ld_any(a.beta, a.beta_dtype, t * a.HV + hv);
            sm.sc[2] = iq;
            sm.sc[3] = ik;
            sm.sc[4] = qk * iq * ik;
            sm.sc[5] = lq;
            sm.sc[6] = lk;
        }
    }
    __syncthreads();
}

template <int NW>
__device__ __forceinline__ float sum_warps(const float (&red)[NW][128], int j) {
    float x = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) x += red[w][j];
    return x;
}

// One forward token on the register state. If o_out != nullptr, warp 0 writes o_t.
template <int NW, bool VEC4, typename TA>
__device__ __forceinline__ void fwd_token(float (&S)[128 / NW][4], TokenSmem<NW>& sm, const RecFwdArgs& a,
                                          TA* o_out) {
    constexpr int RPT = 128 / NW;
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    const float gam = sm.sc[0], bt = sm.sc[1], iq = sm.sc[2], ik = sm.sc[3], kq = sm.sc[4];
    float pk[4] = {0.f, 0.f, 0.f, 0.f}, pq[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int r = 0; r < RPT; ++r) {
        const int i = w + NW * r;
        if (i < a.DK) {
            const float ki = sm.k[i] * ik, qi = sm.q[i] * iq;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                S[r][c] *= gam;
                pk[c] = fmaf(S[r][c], ki, pk[c]);
                pq[c] = fmaf(S[r][c], qi, pq[c]);
            }
        }
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const int j = col_of<VEC4>(l, c);
        if (j < 128) {
            sm.red[0][w][j] = pk[c];
            sm.red[1][w][j] = pq[c];
        }
    }
    __syncthreads();
    float dl[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const int j = col_of<VEC4>(l, c);
        dl[c] = 0.f;
        if (j < a.DV) {
            dl[c] = bt * (sm.v[j] - sum_warps<NW>(sm.red[0], j));
            if (w == 0 && o_out) {
                float val = a.scale * (sum_warps<NW>(sm.red[1], j) + dl[c] * kq);
                if (a.o_mode == 1) val += ld(o_out, j);
                st(o_out, j, val);
            }
        }
    }
#pragma unroll
    for (int r = 0; r < RPT; ++r) {
        const int i = w + NW * r;
        if (i < a.DK) {
            const float ki = sm.k[i] * ik;
#pragma unroll
            for (int c = 0; c < 4; ++c) S[r][c] = fmaf(ki, dl[c], S[r][c]);
        }
    }
}

template <int NW, bool VEC4>
__device__ __forceinline__ void load_state(float (&S)[128 / NW][4], const float* src, int DK, int DV, int identity) {
    constexpr int RPT = 128 / NW;
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
#pragma unroll
    for (int r = 0; r < RPT; ++r) {
        const int i = w + NW * r;
        if (VEC4) {
            float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
            if (i < DK && src) x = *reinterpret_cast<const float4*>(src + (int64_t)i * DV + 4 * l);
            S[r][0] = x.x; S[r][1] = x.y; S[r][2] = x.z; S[r][3] = x.w;
        } else {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int j = col_of<VEC4>(l, c);
                S[r][c] = (i < DK && j < DV && src) ? src[(int64_t)i * DV + j] : 0.f;
            }
        }
        if (identity) {
#pragma unroll
            for (int c = 0; c < 4; ++c) S[r][c] = (i < DK && col_of<VEC4>(l, c) == i) ? 1.f : 0.f;
        }
    }
}

template <int NW, bool VEC4>
__device__ __forceinline__ void store_state(const float (&S)[128 / NW][4], float* dst, int DK, int DV, int acc = 0) {
    constexpr int RPT = 128 / NW;
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
#pragma unroll
    for (int r = 0; r < RPT; ++r) {
        const int i = w + NW * r;
        if (i >= DK) continue;
        if (VEC4) {
            float4* d4 = reinterpret_cast<float4*>(dst + (int64_t)i * DV + 4 * l);
            float4 x = make_float4(S[r][0], S[r][1], S[r][2], S[r][3]);
            if (acc) {
                const float4 y = *d4;
                x.x += y.x; x.y += y.y; x.z += y.z; x.w += y.w;
            }
            *d4 = x;
        } else {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int j = col_of<VEC4>(l, c);
                if (j < DV) dst[(int64_t)i * DV + j] = acc ? dst[(int64_t)i * DV + j] + S[r][c] : S[r][c];
            }
        }
    }
}

constexpr int kFwdWarps = 4;

template <typename TA, bool VEC4>
__global__ void __launch_bounds__(32 * kFwdWarps) rec_fwd_kernel(RecFwdArgs a) {
    constexpr int NW = kFwdWarps;
    __shared__ TokenSmem<NW> sm;
    const int64_t n = blockIdx.x / a.HV;
    const int hv = blockIdx.x % a.HV, hq = hv / (a.HV / a.H);
    int64_t bos, eos;
    seq_bounds(a.cu, a.T, n, bos, eos);
    const int64_t soff = (n * a.HV + hv) * (int64_t)a.DK * a.DV;
    float S[128 / NW][4];
    load_state<NW, VEC4>(S, a.h0 ? a.h0 + soff : nullptr, a.DK, a.DV, a.h0_identity);
    for (int64_t t = bos; t < eos; ++t) {
        load_token<NW, TA>(sm, a, t, hq, hv, nullptr);
        TA* o_t = a.o_mode == 2 ? nullptr : (TA*)a.o + (t * a.HV + hv) * a.DV;
        fwd_token<NW, VEC4, TA>(S, sm, a, o_t);
    }
    if (a.ht) store_state<NW, VEC4>(S, a.ht + soff, a.DK, a.DV, a.ht_accumulate);
}

// ---------------------------------------------------------------------------------------------
// Backward. Per (sequence, value head): a forward sweep stores block-start checkpoints (every
// kRecBlk tokens) in the workspace; then blocks are processed in reverse: the block's states
// S_{t-1} are recomputed into the workspace and the reverse recurrence runs token by token:
//   dH += scale q do^T;  dq = scale S_t do;  ddelta = dH^T k;  dk = dH delta - beta S' ddelta;
//   dv = beta ddelta;  dbeta = ddelta . (v - S'^T k);  dS' = dH - beta k ddelta^T;
//   dg = <dS', S'>;  dH <- exp(g) dS'      (S' = exp(g_t) S_{t-1}, S_t = S' + k delta^T)
// dq/dk are accumulated in fp32 (several value heads may share a q/k head) and converted after.
// ---------------------------------------------------------------------------------------------
constexpr int kRecBlk = 32;
constexpr int kBwdWarps = 8;

struct RecBwdArgs {
    RecFwdArgs f;
    const void* dout;
    const float* dht;
    float *dq_acc, *dk_acc;  // fp32 [tokens, H, DK], zeroed by the host
    void* dv;
    float *dg, *dbeta, *dh0;
    float* ws;          // per-CTA scratch
    int64_t ws_stride;  // floats per CTA
    int64_t nb_max;     // checkpoint slots per CTA
};

template <typename TA, bool VEC4>
__global__ void __launch_bounds__(32 * kBwdWarps) rec_bwd_kernel(RecBwdArgs b) {
    constexpr int NW = kBwdWarps, RPT = 128 / NW;
    __shared__ TokenSmem<NW> sm;
    const RecFwdArgs& a = b.f;
    const int64_t n = blockIdx.x / a.HV;
    const int hv = blockIdx.x % a.HV, hq = hv / (a.HV / a.H);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    int64_t bos, eos;
    seq_bounds(a.cu, a.T, n, bos, eos);
    const int64_t SZ = (int64_t)a.DK * a.DV;
    const int64_t soff = (n * a.HV + hv) * SZ;
    float* ck = b.ws + blockIdx.x * b.ws_stride;
    float* blk = ck + b.nb_max * SZ;
    const int64_t L = eos - bos, nb = (L + kRecBlk - 1) / kRecBlk;

    float S[RPT][4];
    load_state<NW, VEC4>(S, a.h0 ? a.h0 + soff : nullptr, a.DK, a.DV, 0);
    for (int64_t t = bos; t < eos; ++t) {
        if ((t - bos) % kRecBlk == 0) store_state<NW, VEC4>(S, ck + ((t - bos) / kRecBlk) * SZ, a.DK, a.DV);
        load_token<NW, TA>(sm, a, t, hq, hv, nullptr);
        fwd_token<NW, VEC4, TA>(S, sm, a, nullptr);
    }
    float dH[RPT][4];
    load_state<NW, VEC4>(dH, b.dht ? b.dht + soff : nullptr, a.DK, a.DV, 0);

    for (int64_t bi = nb - 1; bi >= 0; --bi) {
        const int64_t t0 = bos + bi * kRecBlk, t1 = min(t0 + kRecBlk, eos);
        load_state<NW, VEC4>(S, ck + bi * SZ, a.DK, a.DV, 0);
        for (int64_t t = t0; t < t1; ++t) {
            // every thread later reads back exactly the slots it stores here: no barrier needed
            store_state<NW, VEC4>(S, blk + (t - t0) * SZ, a.DK, a.DV);
            load_token<NW, TA>(sm, a, t, hq, hv, nullptr);
            fwd_token<NW, VEC4, TA>(S, sm, a, nullptr);
        }
        for (int64_t t = t1 - 1; t >= t0; --t) {
            load_token<NW, TA>(sm, a, t, hq, hv, (const TA*)b.dout);
            const float gam = sm.sc[0], bt = sm.sc[1], iq = sm.sc[2], ik = sm.sc[3];
            float (&Sd)[RPT][4] = S;  // S is free here: reuse its registers for S' = exp(g) S_{t-1}
            load_state<NW, VEC4>(Sd, blk + (t - t0) * SZ, a.DK, a.DV, 0);
            float pk[4] = {0.f, 0.f, 0.f, 0.f}, pd[4] = {0.f, 0.f, 0.f, 0.f};
            float dov[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int j = col_of<VEC4>(l, c);
                dov[c] = j < a.DV ? sm.dout[j] : 0.f;
            }
#pragma unroll
            for (int r = 0; r < RPT; ++r) {
                const int i = w + NW * r;
                if (i < a.DK) {
                    const float ki = sm.k[i] * ik, qi = sm.q[i] * iq;
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        Sd[r][c] *= gam;
                        pk[c] = fmaf(Sd[r][c], ki, pk[c]);
                        dH[r][c] = fmaf(a.scale * qi, dov[c], dH[r][c]);
                        pd[c] = fmaf(dH[r][c], ki, pd[c]);
                    }
                }
            }
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int j = col_of<VEC4>(l, c);
                if (j < 128) {
                    sm.red[0][w][j] = pk[c];
                    sm.red[1][w][j] = pd[c];
                }
            }
            __syncthreads();
            float u[4], dl[4], dd[4];
            float dbp = 0.f;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int j = col_of<VEC4>(l, c);
                u[c] = dl[c] = dd[c] = 0.f;
                if (j < a.DV) {
                    u[c] = sm.v[j] - sum_warps<NW>(sm.red[0], j);
                    dl[c] = bt * u[c];
                    dd[c] = sum_warps<NW>(sm.red[1], j);
                    dbp = fmaf(dd[c], u[c], dbp);
                    if (w == 0) st((TA*)b.dv, (t * a.HV + hv) * a.DV + j, bt * dd[c]);
                }
            }
            dbp = warp_sum(dbp);  // identical in every warp (all columns)
            float dgp = 0.f;
#pragma unroll
            for (int r = 0; r < RPT; ++r) {
                const int i = w + NW * r;
                float xq = 0.f, xk = 0.f;
                const float ki = (i < a.DK) ? sm.k[i] * ik : 0.f;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    xq = fmaf(fmaf(ki, dl[c], Sd[r][c]), dov[c], xq);
                    xk = fmaf(dH[r][c], dl[c], xk);
                    xk = fmaf(-bt * Sd[r][c], dd[c], xk);
                    const float ds = fmaf(-bt * ki, dd[c], dH[r][c]);
                    dgp = fmaf(ds, Sd[r][c], dgp);
                    dH[r][c] = ds * gam;
                }
                xq = warp_sum(xq);
                xk = warp_sum(xk);
                if (l == 0 && i < a.DK) {
                    sm.rowq[i] = a.scale * xq;
                    sm.rowk[i] = xk;
                }
            }
            dgp = warp_sum(dgp);
            if (l == 0) {
                sm.part[w][0] = dgp;
                sm.part[w][1] = dbp;
            }
            __syncthreads();
            // warp 0: dg, dbeta, and the two dot products of the L2-norm chain rule
            if (w == 0) {
                float sq = 0.f, sk = 0.f;
                for (int i = l; i < a.DK; i += 32) {
                    sq += sm.q[i] * iq * sm.rowq[i];
                    sk += sm.k[i] * ik * sm.rowk[i];
                }
                sq = warp_sum(sq);
                sk = warp_sum(sk);
                if (l == 0) {
                    float dgs = 0.f;
#pragma unroll
                    for (int x = 0; x < NW; ++x) dgs += sm.part[x][0];
                    b.dg[t * a.HV + hv] = dgs;
                    b.dbeta[t * a.HV + hv] = sm.part[0][1];
                    sm.sc[7] = sq;
                    sm.part[0][0] = sk;
                }
            }
            __syncthreads();
            if (threadIdx.x < a.DK) {
                const int i = threadIdx.x;
                float gq = sm.rowq[i], gk = sm.rowk[i];
                if (a.l2norm) {
                    const float lq = sm.sc[5], lk = sm.sc[6];
                    gq = (gq - sm.q[i] * iq * sm.sc[7] * (lq > kL2Eps)) * iq;
                    gk = (gk - sm.k[i] * ik * sm.part[0][0] * (lk > kL2Eps)) * ik;
                }
                atomicAdd(b.dq_acc + (t * a.H + hq) * a.DK + i, gq);
                atomicAdd(b.dk_acc + (t * a.H + hq) * a.DK + i, gk);
            }
        }
    }
    if (b.dh0) store_state<NW, VEC4>(dH, b.dh0 + soff, a.DK, a.DV);
}

template <typename TA>
__global__ void convert_kernel(const float* __restrict__ src, TA* __restrict__ dst, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        st(dst, i, src[i]);
}

// ------------------------------------------------------------------------------------------------
// Host launchers
// ------------------------------------------------------------------------------------------------
static RecFwdArgs fwd_args(const RecLaunch& L) {
    RecFwdArgs a{};
    a.q = L.q; a.k = L.k; a.v = L.v; a.g = L.g; a.beta = L.beta;
    a.g_dtype = L.g_dtype; a.beta_dtype = L.beta_dtype;
    a.o = L.o; a.h0 = L.h0; a.ht = L.ht; a.cu = L.cu; a.T = L.T;
    a.H = (int)L.H; a.HV = (int)L.HV; a.DK = (int)L.DK; a.DV = (int)L.DV;
    a.scale = L.scale; a.l2norm = L.l2norm; a.zero_v = L.zero_v; a.o_mode = L.o_mode;
    a.h0_identity = L.h0_identity; a.ht_accumulate = L.ht_accumulate;
    return a;
}

int rec_fwd(const RecLaunch& L, cudaStream_t s) {
    const RecFwdArgs a = fwd_args(L);
    const dim3 grid((unsigned)(L.N * L.HV));
    if (grid.x == 0) return GDN_OK;
    GDN_DISPATCH_DTYPE(L.act_dtype, TA,
        if (a.DV == 128) rec_fwd_kernel<TA, true><<<grid, 32 * kFwdWarps, 0, s>>>(a);
        else rec_fwd_kernel<TA, false><<<grid, 32 * kFwdWarps, 0, s>>>(a);)
    count_launch();
    return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

size_t rec_bwd_workspace(int64_t N, int64_t HV, int64_t DK, int64_t DV, int64_t max_len, int64_t total_tokens,
                         int64_t H) {
    const int64_t nb = (max_len + kRecBlk - 1) / kRecBlk;
    const int64_t per = (nb + kRecBlk) * DK * DV;
    return (size_t)(N * HV * per) * 4 + (size_t)total_tokens * H * DK * 4 * 2 + 256;
}

int rec_bwd(const RecLaunch& L, const void* dout, const float* dht, void* dq, void* dk, void* dv, float* dg,
            float* dbeta, float* dh0, void* ws, int64_t max_len, int64_t total_tokens, cudaStream_t s) {
    RecBwdArgs b;
    RecLaunch Lf = L;
    Lf.o = nullptr; Lf.ht = nullptr; Lf.zero_v = 0; Lf.o_mode = 2; Lf.h0_identity = 0; Lf.ht_accumulate = 0;
    b.f = fwd_args(Lf);
    b.dout = dout;
    b.dht = dht;
    b.dv = dv;
    b.dg = dg;
    b.dbeta = dbeta;
    b.dh0 = dh0;
    b.nb_max = (max_len + kRecBlk - 1) / kRecBlk;
    b.ws_stride = (b.nb_max + kRecBlk) * L.DK * L.DV;
    char* base = (char*)ws + 256;
    b.dq_acc = (float*)base;
    b.dk_acc = b.dq_acc + total_tokens * L.H * L.DK;
    b.ws = b.dk_acc + total_tokens * L.H * L.DK;
    const int64_t nqk = total_tokens * L.H * L.DK;
    if (nqk > 0 && cudaMemsetAsync(b.dq_acc, 0, sizeof(float) * nqk * 2, s) != cudaSuccess) return GDN_ERR_LAUNCH;
    const dim3 grid((unsigned)(L.N * L.HV));
    if (grid.x > 0) {
        GDN_DISPATCH_DTYPE(L.act_dtype, TA,
            if (b.f.DV == 128) rec_bwd_kernel<TA, true><<<grid, 32 * kBwdWarps, 0, s>>>(b);
            else rec_bwd_kernel<TA, false><<<grid, 32 * kBwdWarps, 0, s>>>(b);)
        count_launch();
    }
    if (nqk > 0) {
        const int64_t want = (nqk + 255) / 256;
        const unsigned blocks = (unsigned)(want < 148 * 16 ? want : 148 * 16);
        GDN_DISPATCH_DTYPE(L.act_dtype, TA,
            convert_kernel<TA><<<blocks, 256, 0, s>>>(b.dq_acc, (TA*)dq, nqk);
            convert_kernel<TA><<<blocks, 256, 0, s>>>(b.dk_acc, (TA*)dk, nqk);)
        count_launch(2);
    }
    return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

}  // namespace gdn
