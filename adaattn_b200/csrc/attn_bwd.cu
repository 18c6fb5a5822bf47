// Attention backward on the CUDA cores (FFMA, fp32 arithmetic).
//
// The reference's AdaAttention is differentiable through ATen autograd
// (tests/unit/test_adaattn_unified.py:146-159). These kernels give the
// gradients of the attention function each head evaluates,
//   out = softmax(q k^T * scale + mask) v       (dense heads; low-rank heads
//   pass q_low = q W^T, k_low = k W^T as q, k, and the caller chains W),
// in fp32 at the operands' values, recomputing the probabilities from a
// per-row log-sum-exp instead of storing them:
//   prep:  LSE_i = log sum_j exp(z_ij), Delta_i = sum_d dO_id O_id
//   main:  one CTA per (b, h, 64-key block j), looping over query blocks i:
//          P = exp(z - LSE), dV_j += P^T dO_i, dP = dO_i V_j^T,
//          dS = P (dP - Delta_i), dK_j += scale dS^T Q_i,
//          dQ_i += scale dS K_j (fp32 atomics across key blocks).
// Causal masking is top-left aligned (key c hidden from query r when c > r);
// bool masks hide keys, float masks are added to z, as in the forward.
// Thread (ty, tx) of 256 owns rows 4*ty..4*ty+3 and columns tx + 16*c of a
// 64 x 64 score tile, and output columns 64*g + 4*tx + e of 4 rows of the
// dK / dV / dQ tiles; every operand fetch is a 16-byte shared load.
#include "ada_common.cuh"
#include "ada_internal.h"

namespace ada {
namespace {

constexpr int kB = 64;          // query and key rows per tile
constexpr int kT = 256;
constexpr int kLdS = kB + 4;    // score / P / dS tiles

template <int DQKP, int DVP>
struct BwdCfg {
    static constexpr int LDQ = DQKP + 4;
    static constexpr int LDV = DVP + 4;
    static constexpr int GQ = DQKP / 64;
    static constexpr int GV = DVP / 64;
    // K, V, Q, dO tiles + P and dS tiles + per-row LSE and Delta
    static constexpr size_t SMEM =
        (static_cast<size_t>(kB) * LDQ * 2 + static_cast<size_t>(kB) * LDV * 2 + static_cast<size_t>(kB) * kLdS * 2 +
         2 * kB) *
        sizeof(float);
};

// rows [row0, row0 + 64) x [0, w) of a [.., N, w] view into a padded shared
// tile (zeros past n or w).
__device__ __forceinline__ void stage_rows(float* dst, int ld, int width_p, const void* src, int dtype, int64_t base,
                                           int64_t s_row, int64_t s_col, int64_t row0, int64_t n, int w) {
    for (int idx = threadIdx.x; idx < kB * width_p; idx += kT) {
        const int r = idx / width_p, c = idx - r * width_p;
        const int64_t row = row0 + r;
        dst[r * ld + c] = (row < n && c < w) ? load_as_f32(src, base + row * s_row + c * s_col, dtype) : 0.f;
    }
}

__device__ __forceinline__ bool key_visible(const BwdLaunch& L, int64_t b, int64_t h, int64_t row, int64_t col,
                                            float& add) {
    add = 0.f;
    if (row >= L.Nq || col >= L.Nk) return false;
    if (L.causal && col > row) return false;
    if (L.mask.data != nullptr) {
        const int64_t off = b * L.mask.s[0] + h * L.mask.s[1] + row * L.mask.s[2] + col * L.mask.s[3];
        const float m = load_as_f32(L.mask.data, off, L.mask.dtype);
        if (L.mask.dtype == ADA_BOOL) {
            if (m == 0.f) return false;
        } else {
            add = m;
        }
    }
    return true;
}

// 4 x 4 block of A B^T over `width` columns: rows 4*ty + i of A, rows tx + 16*j of B.
__device__ __forceinline__ void block_abt(const float* A, int lda, const float* Bm, int ldb, int width, int ty, int tx,
                                          float (&acc)[4][4]) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
    for (int d = 0; d < width; d += 4) {
        float4 a[4], bb[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) a[i] = *reinterpret_cast<const float4*>(A + (4 * ty + i) * lda + d);
#pragma unroll
        for (int j = 0; j < 4; ++j) bb[j] = *reinterpret_cast<const float4*>(Bm + (tx + 16 * j) * ldb + d);
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                acc[i][j] = fmaf(a[i].x, bb[j].x, acc[i][j]);
                acc[i][j] = fmaf(a[i].y, bb[j].y, acc[i][j]);
                acc[i][j] = fmaf(a[i].z, bb[j].z, acc[i][j]);
                acc[i][j] = fmaf(a[i].w, bb[j].w, acc[i][j]);
            }
    }
}

template <int DQKP, int DVP>
__global__ void __launch_bounds__(kT) attn_bwd_prep_kernel(const __grid_constant__ BwdLaunch L) {
    using C = BwdCfg<DQKP, DVP>;
    extern __shared__ __align__(16) float sm[];
    float* sQ = sm;
    float* sK = sQ + kB * C::LDQ;
    const int64_t bh = blockIdx.y;
    if (!head_selected(L.sel, bh)) return;
    const int64_t b = bh / L.H, h = bh % L.H;
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    const int64_t q0 = static_cast<int64_t>(blockIdx.x) * kB;
    stage_rows(sQ, C::LDQ, DQKP, L.q, L.q_dtype, b * L.qs[0] + h * L.qs[1], L.qs[2], L.qs[3], q0, L.Nq, L.dqk);
    float m[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.f;
    }
    const int64_t n_kb = (L.Nk + kB - 1) / kB;
    for (int64_t kb = 0; kb < n_kb; ++kb) {
        const int64_t k0 = kb * kB;
        if (L.causal && k0 > q0 + kB - 1) break;
        __syncthreads();
        stage_rows(sK, C::LDQ, DQKP, L.k, L.k_dtype, b * L.ks[0] + h * L.ks[1], L.ks[2], L.ks[3], k0, L.Nk, L.dqk);
        __syncthreads();
        float acc[4][4];
        block_abt(sQ, C::LDQ, sK, C::LDQ, DQKP, ty, tx, acc);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float z[4];
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float add;
                const bool ok = key_visible(L, b, h, q0 + 4 * ty + i, k0 + tx + 16 * j, add);
                z[j] = ok ? acc[i][j] * L.scale + add : -INFINITY;
                mx = fmaxf(mx, z[j]);
            }
            for (int o = 8; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            const float m_new = fmaxf(m[i], mx);
            float s = 0.f;
            if (m_new != -INFINITY) {
#pragma unroll
                for (int j = 0; j < 4; ++j) s += (z[j] == -INFINITY) ? 0.f : expf(z[j] - m_new);
            }
            for (int o = 8; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            l[i] = (m_new == -INFINITY) ? 0.f : l[i] * ((m[i] == -INFINITY) ? 0.f : expf(m[i] - m_new)) + s;
            m[i] = m_new;
        }
    }
    // Delta_i = sum_d dO_id * O_id over the value width
    const int64_t obase = b * L.os[0] + h * L.os[1];
    const int64_t gbase = b * L.gs[0] + h * L.gs[1];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t row = q0 + 4 * ty + i;
        float dsum = 0.f;
        if (row < L.Nq)
            for (int d = tx; d < L.dv; d += 16)
                dsum += load_as_f32(L.dout, gbase + row * L.gs[2] + d * L.gs[3], L.dout_dtype) *
                        load_as_f32(L.out, obase + row * L.os[2] + d * L.os[3], L.out_dtype);
        for (int o = 8; o > 0; o >>= 1) dsum += __shfl_xor_sync(0xffffffffu, dsum, o);
        if (tx == 0 && row < L.Nq) {
            // A row with no visible key has no probabilities: +inf makes every P 0.
            L.lse[bh * L.Nq + row] = (l[i] > 0.f) ? m[i] + logf(l[i]) : INFINITY;
            L.delta[bh * L.Nq + row] = dsum;
        }
    }
}

template <int DQKP, int DVP>
__global__ void __launch_bounds__(kT) attn_bwd_main_kernel(const __grid_constant__ BwdLaunch L) {
    using C = BwdCfg<DQKP, DVP>;
    extern __shared__ __align__(16) float sm[];
    float* sK = sm;
    float* sQ = sK + kB * C::LDQ;
    float* sV = sQ + kB * C::LDQ;
    float* sdO = sV + kB * C::LDV;
    float* sP = sdO + kB * C::LDV;
    float* sdS = sP + kB * kLdS;
    float* sLse = sdS + kB * kLdS;
    float* sDelta = sLse + kB;
    const int64_t bh = blockIdx.y;
    if (!head_selected(L.sel, bh)) return;
    const int64_t b = bh / L.H, h = bh % L.H;
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    const int64_t k0 = static_cast<int64_t>(blockIdx.x) * kB;
    const float scale = L.scale;
    stage_rows(sK, C::LDQ, DQKP, L.k, L.k_dtype, b * L.ks[0] + h * L.ks[1], L.ks[2], L.ks[3], k0, L.Nk, L.dqk);
    stage_rows(sV, C::LDV, DVP, L.v, L.v_dtype, b * L.vs[0] + h * L.vs[1], L.vs[2], L.vs[3], k0, L.Nk, L.dv);
    float dk[4][4 * C::GQ], dv[4][4 * C::GV];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
        for (int c = 0; c < 4 * C::GQ; ++c) dk[i][c] = 0.f;
#pragma unroll
        for (int c = 0; c < 4 * C::GV; ++c) dv[i][c] = 0.f;
    }
    const int64_t n_qb = (L.Nq + kB - 1) / kB;
    // Top-left causal alignment: query block i sees key block j only when i >= j.
    const int64_t qb0 = L.causal ? blockIdx.x : 0;
    for (int64_t qb = qb0; qb < n_qb; ++qb) {
        const int64_t q0 = qb * kB;
        __syncthreads();
        stage_rows(sQ, C::LDQ, DQKP, L.q, L.q_dtype, b * L.qs[0] + h * L.qs[1], L.qs[2], L.qs[3], q0, L.Nq, L.dqk);
        stage_rows(sdO, C::LDV, DVP, L.dout, L.dout_dtype, b * L.gs[0] + h * L.gs[1], L.gs[2], L.gs[3], q0, L.Nq,
                   L.dv);
        if (tid < kB) {
            const int64_t row = q0 + tid;
            sLse[tid] = row < L.Nq ? L.lse[bh * L.Nq + row] : INFINITY;
            sDelta[tid] = row < L.Nq ? L.delta[bh * L.Nq + row] : 0.f;
        }
        __syncthreads();
        // P = exp(z - LSE) and dS = P (dO V^T - Delta), 4 x 4 per thread
        float s[4][4], dp[4][4];
        block_abt(sQ, C::LDQ, sK, C::LDQ, DQKP, ty, tx, s);
        block_abt(sdO, C::LDV, sV, C::LDV, DVP, ty, tx, dp);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int r = 4 * ty + i;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int c = tx + 16 * j;
                float add;
                const bool ok = key_visible(L, b, h, q0 + r, k0 + c, add);
                const float p = ok ? expf(s[i][j] * scale + add - sLse[r]) : 0.f;
                sP[r * kLdS + c] = p;
                sdS[r * kLdS + c] = p * (dp[i][j] - sDelta[r]);
            }
        }
        __syncthreads();
        // dV_j += P^T dO_i and dK_j += dS^T Q_i: keys 4*ty + kk, columns 64*g + 4*tx + e
        for (int r = 0; r < kB; ++r) {
            const float4 pk = *reinterpret_cast<const float4*>(sP + r * kLdS + 4 * ty);
            const float4 sk = *reinterpret_cast<const float4*>(sdS + r * kLdS + 4 * ty);
            const float pa[4] = {pk.x, pk.y, pk.z, pk.w};
            const float sa[4] = {sk.x, sk.y, sk.z, sk.w};
#pragma unroll
            for (int g = 0; g < C::GV; ++g) {
                const float4 o = *reinterpret_cast<const float4*>(sdO + r * C::LDV + 64 * g + 4 * tx);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    dv[kk][4 * g + 0] = fmaf(pa[kk], o.x, dv[kk][4 * g + 0]);
                    dv[kk][4 * g + 1] = fmaf(pa[kk], o.y, dv[kk][4 * g + 1]);
                    dv[kk][4 * g + 2] = fmaf(pa[kk], o.z, dv[kk][4 * g + 2]);
                    dv[kk][4 * g + 3] = fmaf(pa[kk], o.w, dv[kk][4 * g + 3]);
                }
            }
#pragma unroll
            for (int g = 0; g < C::GQ; ++g) {
                const float4 qv = *reinterpret_cast<const float4*>(sQ + r * C::LDQ + 64 * g + 4 * tx);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    dk[kk][4 * g + 0] = fmaf(sa[kk], qv.x, dk[kk][4 * g + 0]);
                    dk[kk][4 * g + 1] = fmaf(sa[kk], qv.y, dk[kk][4 * g + 1]);
                    dk[kk][4 * g + 2] = fmaf(sa[kk], qv.z, dk[kk][4 * g + 2]);
                    dk[kk][4 * g + 3] = fmaf(sa[kk], qv.w, dk[kk][4 * g + 3]);
                }
            }
        }
        // dQ_i += scale * dS K_j: rows 4*ty + i, columns 64*g + 4*tx + e
        float dq[4][4 * C::GQ];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int c = 0; c < 4 * C::GQ; ++c) dq[i][c] = 0.f;
        for (int c = 0; c < kB; ++c) {
            float sa[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) sa[i] = sdS[(4 * ty + i) * kLdS + c];
#pragma unroll
            for (int g = 0; g < C::GQ; ++g) {
                const float4 kv = *reinterpret_cast<const float4*>(sK + c * C::LDQ + 64 * g + 4 * tx);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    dq[i][4 * g + 0] = fmaf(sa[i], kv.x, dq[i][4 * g + 0]);
                    dq[i][4 * g + 1] = fmaf(sa[i], kv.y, dq[i][4 * g + 1]);
                    dq[i][4 * g + 2] = fmaf(sa[i], kv.z, dq[i][4 * g + 2]);
                    dq[i][4 * g + 3] = fmaf(sa[i], kv.w, dq[i][4 * g + 3]);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int64_t row = q0 + 4 * ty + i;
            if (row >= L.Nq) continue;
            float* dst = L.dq + (bh * L.Nq + row) * L.dqk;
#pragma unroll
            for (int g = 0; g < C::GQ; ++g)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int col = 64 * g + 4 * tx + e;
                    if (col < L.dqk) atomicAdd(dst + col, scale * dq[i][4 * g + e]);
                }
        }
    }
    // this CTA's key rows of dK (scaled) and dV
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
        const int64_t key = k0 + 4 * ty + kk;
        if (key >= L.Nk) continue;
#pragma unroll
        for (int g = 0; g < C::GQ; ++g)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int col = 64 * g + 4 * tx + e;
                if (col < L.dqk) L.dk[(bh * L.Nk + key) * L.dqk + col] = scale * dk[kk][4 * g + e];
            }
#pragma unroll
        for (int g = 0; g < C::GV; ++g)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int col = 64 * g + 4 * tx + e;
                if (col < L.dv) L.dv_out[(bh * L.Nk + key) * L.dv + col] = dv[kk][4 * g + e];
            }
    }
}

template <int DQKP, int DVP>
int launch_bwd_variant(const BwdLaunch& L, cudaStream_t stream) {
    using C = BwdCfg<DQKP, DVP>;
    const size_t smem = C::SMEM;
    if (cudaFuncSetAttribute(attn_bwd_prep_kernel<DQKP, DVP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess ||
        cudaFuncSetAttribute(attn_bwd_main_kernel<DQKP, DVP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
        return ADA_ERR_LAUNCH;
    const int64_t BH = L.B * L.H;
    const int64_t nqb = (L.Nq + kB - 1) / kB, nkb = (L.Nk + kB - 1) / kB;
    if (BH == 0 || nqb == 0 || nkb == 0) return ADA_OK;
    attn_bwd_prep_kernel<DQKP, DVP>
        <<<dim3(static_cast<unsigned>(nqb), static_cast<unsigned>(BH)), kT, smem, stream>>>(L);
    if (cudaGetLastError() != cudaSuccess) return ADA_ERR_LAUNCH;
    attn_bwd_main_kernel<DQKP, DVP>
        <<<dim3(static_cast<unsigned>(nkb), static_cast<unsigned>(BH)), kT, smem, stream>>>(L);
    return cudaGetLastError() == cudaSuccess ? ADA_OK : ADA_ERR_LAUNCH;
}

}  // namespace

int launch_attn_bwd(const BwdLaunch& L, cudaStream_t stream) {
    const int qp = L.dqk <= 64 ? 64 : 128;
    const int vp = L.dv <= 64 ? 64 : 128;
    if (L.dqk > 128 || L.dv > 128) return ADA_ERR_UNSUPPORTED;
    if (qp == 64 && vp == 64) return launch_bwd_variant<64, 64>(L, stream);
    if (qp == 64 && vp == 128) return launch_bwd_variant<64, 128>(L, stream);
    if (qp == 128 && vp == 64) return launch_bwd_variant<128, 64>(L, stream);
    return launch_bwd_variant<128, 128>(L, stream);
}

}  // namespace ada
