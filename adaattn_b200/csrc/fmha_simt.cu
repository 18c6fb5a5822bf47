// FP32 heads: fused attention forward on the CUDA cores (FFMA), the
// non-tensor-core path for heads whose decision is FP32 (adaattn.py:300-339
// with target dtype float32, and the low-rank branch :341-394 on q_low/k_low).
//
// A CTA owns 64 query rows of one (b, h); 256 threads as 16 x 16. Key/value
// blocks of 64 rows are staged in shared memory (K transposed), scores and
// the online softmax stay in registers, exp is expf (full fp32 accuracy).
// Thread (ty, tx) owns query rows 4*ty..4*ty+3, score columns tx + 16*i and
// output columns tx + 16*i: strided ownership keeps shared loads conflict free.
#include "ada_common.cuh"
#include "ada_internal.h"

namespace ada {
namespace {

constexpr int kBQ = 64;
constexpr int kBK = 64;
constexpr int kDMax = 128;
constexpr int kThreadsS = 256;
constexpr int kLdKt = kBK + 1;

__global__ void __launch_bounds__(kThreadsS) fmha_simt_kernel(const __grid_constant__ SimtLaunch L) {
    extern __shared__ float sm[];
    float* sQ = sm;                          // [kBQ][dqk]
    float* sKt = sQ + kBQ * kDMax;           // [dqk][kLdKt]
    float* sV = sKt + kDMax * kLdKt;         // [kBK][dv]
    float* sP = sV + kBK * kDMax;            // [kBQ][kBK + 1]

    const int64_t BH = L.B * L.H;
    const int64_t nqb = (L.Nq + kBQ - 1) / kBQ;
    const int64_t lin = blockIdx.x;
    const int64_t bh = lin % BH;
    const int64_t qb = nqb - 1 - lin / BH;
    if (!head_selected(L.sel, bh)) return;
    const int64_t b = bh / L.H, h = bh % L.H;
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    const int dqk = L.dqk, dv = L.dv;
    const int64_t q0 = qb * kBQ;

    {
        const int64_t base = b * L.qs[0] + h * L.qs[1];
        for (int i = tid; i < kBQ * dqk; i += kThreadsS) {
            const int r = i / dqk, d = i - r * dqk;
            const int64_t row = q0 + r;
            sQ[r * dqk + d] = row < L.Nq ? load_as_f32(L.q, base + row * L.qs[2] + d * L.qs[3], L.q_dtype) : 0.f;
        }
    }
    float m[4], l[4], o[4][8];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        m[r] = -INFINITY;
        l[r] = 0.f;
#pragma unroll
        for (int c = 0; c < 8; ++c) o[r][c] = 0.f;
    }
    int64_t nkb = (L.Nk + kBK - 1) / kBK;
    if (L.causal) {
        const int64_t last = (q0 + kBQ - 1 < L.Nq - 1 ? q0 + kBQ - 1 : L.Nq - 1);
        const int64_t need = last / kBK + 1;
        if (need < nkb) nkb = need;
    }
    const int64_t kbase = b * L.ks[0] + h * L.ks[1];
    const int64_t vbase = b * L.vs[0] + h * L.vs[1];
    for (int64_t kb = 0; kb < nkb; ++kb) {
        const int64_t k0 = kb * kBK;
        __syncthreads();
        for (int i = tid; i < kBK * dqk; i += kThreadsS) {
            const int r = i / dqk, d = i - r * dqk;
            const int64_t row = k0 + r;
            sKt[d * kLdKt + r] = row < L.Nk ? load_as_f32(L.k, kbase + row * L.ks[2] + d * L.ks[3], L.k_dtype) : 0.f;
        }
        for (int i = tid; i < kBK * dv; i += kThreadsS) {
            const int r = i / dv, d = i - r * dv;
            const int64_t row = k0 + r;
            sV[r * dv + d] = row < L.Nk ? load_as_f32(L.v, vbase + row * L.vs[2] + d * L.vs[3], L.v_dtype) : 0.f;
        }
        __syncthreads();
        float s[4][4];
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int i = 0; i < 4; ++i) s[r][i] = 0.f;
        for (int d = 0; d < dqk; ++d) {
            float a[4], kk[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) a[r] = sQ[(ty * 4 + r) * dqk + d];
#pragma unroll
            for (int i = 0; i < 4; ++i) kk[i] = sKt[d * kLdKt + tx + 16 * i];
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int i = 0; i < 4; ++i) s[r][i] = fmaf(a[r], kk[i], s[r][i]);
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int64_t qrow = q0 + ty * 4 + r;
            float mx = -INFINITY;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int64_t kv = k0 + tx + 16 * i;
                float v = s[r][i] * L.scale;
                if (kv >= L.Nk || (L.causal && kv > qrow)) v = -INFINITY;
                if (L.mask.data != nullptr && kv < L.Nk && qrow < L.Nq) {
                    const float mv = load_as_f32(L.mask.data,
                                                 b * L.mask.s[0] + h * L.mask.s[1] + qrow * L.mask.s[2] +
                                                     kv * L.mask.s[3],
                                                 L.mask.dtype);
                    if (L.mask.dtype == ADA_BOOL) {
                        if (mv == 0.f) v = -INFINITY;
                    } else {
                        v += mv;
                    }
                }
                s[r][i] = v;
                mx = fmaxf(mx, v);
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float m_new = fmaxf(m[r], mx);
            const float alpha = (m_new == -INFINITY) ? 1.f : expf(m[r] - m_new);
            float sum = 0.f;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float p = (m_new == -INFINITY) ? 0.f : expf(s[r][i] - m_new);
                s[r][i] = p;
                sum += p;
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
            l[r] = l[r] * alpha + sum;
            m[r] = m_new;
#pragma unroll
            for (int c = 0; c < 8; ++c) o[r][c] *= alpha;
#pragma unroll
            for (int i = 0; i < 4; ++i) sP[(ty * 4 + r) * (kBK + 1) + tx + 16 * i] = s[r][i];
        }
        __syncthreads();
        for (int c = 0; c < kBK; ++c) {
            float p[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) p[r] = sP[(ty * 4 + r) * (kBK + 1) + c];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int col = tx + 16 * j;
                const float vv = col < dv ? sV[c * dv + col] : 0.f;
#pragma unroll
                for (int r = 0; r < 4; ++r) o[r][j] = fmaf(p[r], vv, o[r][j]);
            }
        }
    }
    const int64_t obase = b * L.os[0] + h * L.os[1];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const int64_t qrow = q0 + ty * 4 + r;
        if (qrow >= L.Nq) continue;
        const float inv = 1.f / l[r];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int col = tx + 16 * j;
            if (col < dv) store_from_f32(L.out, obase + qrow * L.os[2] + col * L.os[3], L.out_dtype, o[r][j] * inv);
        }
    }
}

}  // namespace

int launch_fmha_simt(const SimtLaunch& L, cudaStream_t stream) {
    if (L.dqk > kDMax || L.dv > kDMax || L.dqk <= 0 || L.dv <= 0) return ADA_ERR_UNSUPPORTED;
    const size_t smem = (static_cast<size_t>(kBQ) * kDMax + static_cast<size_t>(kDMax) * kLdKt +
                         static_cast<size_t>(kBK) * kDMax + static_cast<size_t>(kBQ) * (kBK + 1)) *
                        sizeof(float);
    if (cudaFuncSetAttribute(fmha_simt_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
        return ADA_ERR_LAUNCH;
    const int64_t nqb = (L.Nq + kBQ - 1) / kBQ;
    const int64_t grid = nqb * L.B * L.H;
    if (grid <= 0) return ADA_OK;
    if (grid > 0x7fffffffLL) return ADA_ERR_UNSUPPORTED;
    fmha_simt_kernel<<<static_cast<unsigned>(grid), kThreadsS, smem, stream>>>(L);
    return cudaGetLastError() == cudaSuccess ? ADA_OK : ADA_ERR_LAUNCH;
}

}  // namespace ada
