// FP32 heads: fused attention forward on the CUDA cores (FFMA), the
// non-tensor-core path for heads whose decision is FP32 (adaattn.py:300-339
// with target dtype float32, and the low-rank branch :341-394 on q_low/k_low).
//
// A CTA owns 64 query rows of one (b, h); 256 threads as 16 x 16. Key/value
// blocks of 64 rows are staged in shared memory, scores and the online
// softmax stay in registers, exp is expf (full fp32 accuracy).
// Thread (ty, tx) owns query rows 4*ty..4*ty+3, score columns tx + 16*i and
// output columns 64*g + 4*tx + e. Every operand fetch is a 16-byte shared
// load (rows padded by 16 bytes, so the 8 rows or 16 keys a warp touches at
// once fall in distinct banks): Q.K^T takes 8 such loads per 64 FMAs, P.V
// 4 + 4*G per 64*G FMAs.
#include "ada_common.cuh"
#include "ada_internal.h"

namespace ada {
namespace {

constexpr int kBQ = 64;
constexpr int kBK = 64;
constexpr int kThreadsS = 256;
constexpr int kLdP = kBK + 4;

template <int DQKP, int DVP>
struct SimtCfg {
    static constexpr int LDQ = DQKP + 4;  // Q and K rows
    static constexpr int LDV = DVP + 4;
    static constexpr int G = DVP / 64;    // 4-column output groups per thread
    static constexpr size_t SMEM =
        (static_cast<size_t>(2) * kBQ * LDQ + static_cast<size_t>(kBK) * LDV + static_cast<size_t>(kBQ) * kLdP) *
        sizeof(float);
};

// rows [row0, row0 + 64) x [0, width) of a [.., N, w] view into a padded
// shared tile (zeros past n or w); 4 columns per step, 16-byte global loads
// when the view allows them.
__device__ __forceinline__ void load_tile(float* dst, int ld, int width_p, const void* src, int dtype,
                                          int64_t base, int64_t s_row, int64_t s_col, int64_t row0, int64_t n,
                                          int w, bool vec) {
    const int groups = width_p / 4;
    for (int idx = threadIdx.x; idx < kBK * groups; idx += kThreadsS) {
        const int r = idx / groups, c0 = (idx - r * groups) * 4;
        const int64_t row = row0 + r;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (row < n) {
            const int64_t e = base + row * s_row + c0 * s_col;
            if (vec && c0 + 4 <= w) {
                if (dtype == ADA_F32) {
                    v = *reinterpret_cast<const float4*>(static_cast<const float*>(src) + e);
                } else {
                    const uint2 u = *reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(src) + e);
                    if (dtype == ADA_BF16) {
                        const __nv_bfloat162 lo = *reinterpret_cast<const __nv_bfloat162*>(&u.x);
                        const __nv_bfloat162 hi = *reinterpret_cast<const __nv_bfloat162*>(&u.y);
                        v = make_float4(__low2float(lo), __high2float(lo), __low2float(hi), __high2float(hi));
                    } else {
                        const __half2 lo = *reinterpret_cast<const __half2*>(&u.x);
                        const __half2 hi = *reinterpret_cast<const __half2*>(&u.y);
                        v = make_float4(__low2float(lo), __high2float(lo), __low2float(hi), __high2float(hi));
                    }
                }
            } else {
                float t[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) t[k] = (c0 + k < w) ? load_as_f32(src, e + k * s_col, dtype) : 0.f;
                v = make_float4(t[0], t[1], t[2], t[3]);
            }
        }
        *reinterpret_cast<float4*>(dst + r * ld + c0) = v;
    }
}

// 16-byte (fp32) or 8-byte (16-bit) vector loads of 4 elements stay aligned.
__device__ __forceinline__ bool vec_ok(const void* p, int dtype, const int64_t* st) {
    if (dtype != ADA_F32 && dtype != ADA_F16 && dtype != ADA_BF16) return false;
    const int eb = dtype == ADA_F32 ? 4 : 2;
    const int need = 4 * eb;
    if (st[3] != 1) return false;
    if ((reinterpret_cast<uintptr_t>(p) & 15u) != 0) return false;
    for (int i = 0; i < 3; ++i)
        if (((st[i] * eb) % need) != 0) return false;
    return true;
}

template <int DQKP, int DVP>
__global__ void __launch_bounds__(kThreadsS, 2) fmha_simt_kernel(const __grid_constant__ SimtLaunch L) {
    using C = SimtCfg<DQKP, DVP>;
    extern __shared__ float sm[];
    float* sQ = sm;                     // [kBQ][LDQ]
    float* sK = sQ + kBQ * C::LDQ;      // [kBK][LDQ]
    float* sV = sK + kBK * C::LDQ;      // [kBK][LDV]
    float* sP = sV + kBK * C::LDV;      // [kBQ][kLdP]

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
    const bool vq = vec_ok(L.q, L.q_dtype, L.qs);
    const bool vk = vec_ok(L.k, L.k_dtype, L.ks);
    const bool vv = vec_ok(L.v, L.v_dtype, L.vs);

    load_tile(sQ, C::LDQ, DQKP, L.q, L.q_dtype, b * L.qs[0] + h * L.qs[1], L.qs[2], L.qs[3], q0, L.Nq, dqk, vq);
    float m[4], l[4], o[4][4 * C::G];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        m[r] = -INFINITY;
        l[r] = 0.f;
#pragma unroll
        for (int c = 0; c < 4 * C::G; ++c) o[r][c] = 0.f;
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
        load_tile(sK, C::LDQ, DQKP, L.k, L.k_dtype, kbase, L.ks[2], L.ks[3], k0, L.Nk, dqk, vk);
        load_tile(sV, C::LDV, DVP, L.v, L.v_dtype, vbase, L.vs[2], L.vs[3], k0, L.Nk, dv, vv);
        __syncthreads();
        float s[4][4];
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int i = 0; i < 4; ++i) s[r][i] = 0.f;
#pragma unroll 4
        for (int d = 0; d < DQKP; d += 4) {
            float4 a[4], kk[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) a[r] = *reinterpret_cast<const float4*>(sQ + (ty * 4 + r) * C::LDQ + d);
#pragma unroll
            for (int i = 0; i < 4; ++i) kk[i] = *reinterpret_cast<const float4*>(sK + (tx + 16 * i) * C::LDQ + d);
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    s[r][i] = fmaf(a[r].x, kk[i].x, s[r][i]);
                    s[r][i] = fmaf(a[r].y, kk[i].y, s[r][i]);
                    s[r][i] = fmaf(a[r].z, kk[i].z, s[r][i]);
                    s[r][i] = fmaf(a[r].w, kk[i].w, s[r][i]);
                }
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
            for (int c = 0; c < 4 * C::G; ++c) o[r][c] *= alpha;
#pragma unroll
            for (int i = 0; i < 4; ++i) sP[(ty * 4 + r) * kLdP + tx + 16 * i] = s[r][i];
        }
        __syncthreads();
#pragma unroll 2
        for (int c = 0; c < kBK; c += 4) {
            float4 p[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) p[r] = *reinterpret_cast<const float4*>(sP + (ty * 4 + r) * kLdP + c);
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
#pragma unroll
                for (int g = 0; g < C::G; ++g) {
                    const float4 v = *reinterpret_cast<const float4*>(sV + (c + cc) * C::LDV + 64 * g + 4 * tx);
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        const float pr = cc == 0 ? p[r].x : cc == 1 ? p[r].y : cc == 2 ? p[r].z : p[r].w;
                        o[r][4 * g + 0] = fmaf(pr, v.x, o[r][4 * g + 0]);
                        o[r][4 * g + 1] = fmaf(pr, v.y, o[r][4 * g + 1]);
                        o[r][4 * g + 2] = fmaf(pr, v.z, o[r][4 * g + 2]);
                        o[r][4 * g + 3] = fmaf(pr, v.w, o[r][4 * g + 3]);
                    }
                }
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
        for (int g = 0; g < C::G; ++g)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int col = 64 * g + 4 * tx + e;
                if (col < dv)
                    store_from_f32(L.out, obase + qrow * L.os[2] + col * L.os[3], L.out_dtype, o[r][4 * g + e] * inv);
            }
    }
}

// ---------------------------------------------------------------------------
// Pipelined variant: K (fp32) and V (fp32 or 16-bit, kept in its own width in
// shared memory) stream through double buffers with cp.async, so block j+1
// is in flight while block j is computed. Used when K is fp32 and both K and
// V rows are 16-byte aligned with widths that are whole 16-byte chunks.
// ---------------------------------------------------------------------------
template <int DQKP, int DVP, int VT>  // VT: element type of V in shared memory (ADA_F32 / ADA_F16 / ADA_BF16)
struct AsyncCfg {
    static constexpr int LDQ = DQKP + 4;               // fp32 Q and K rows
    static constexpr int VEB = VT == ADA_F32 ? 4 : 2;  // bytes per V element
    static constexpr int LDV = DVP + 16 / VEB;         // V row, padded by 16 bytes
    static constexpr int G = DVP / 64;
    static constexpr size_t Q_BYTES = static_cast<size_t>(kBQ) * LDQ * 4;
    static constexpr size_t K_BYTES = static_cast<size_t>(kBK) * LDQ * 4;
    static constexpr size_t V_BYTES = static_cast<size_t>(kBK) * LDV * VEB;
    static constexpr size_t P_BYTES = static_cast<size_t>(kBQ) * kLdP * 4;
    static constexpr size_t SMEM = Q_BYTES + 2 * K_BYTES + 2 * V_BYTES + P_BYTES;
};

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem_dst)), "l"(gsrc),
                 "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// 4 consecutive V elements of row `row` starting at column `col`, as fp32.
template <int VT>
__device__ __forceinline__ float4 v4(const uint8_t* sV, int ldv, int row, int col) {
    if constexpr (VT == ADA_F32) {
        return *reinterpret_cast<const float4*>(sV + (static_cast<size_t>(row) * ldv + col) * 4);
    } else {
        const uint2 u = *reinterpret_cast<const uint2*>(sV + (static_cast<size_t>(row) * ldv + col) * 2);
        if constexpr (VT == ADA_BF16) {
            return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u),
                               __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));
        } else {
            const __half2 lo = *reinterpret_cast<const __half2*>(&u.x);
            const __half2 hi = *reinterpret_cast<const __half2*>(&u.y);
            return make_float4(__low2float(lo), __high2float(lo), __low2float(hi), __high2float(hi));
        }
    }
}

template <int DQKP, int DVP, int VT>
__global__ void __launch_bounds__(kThreadsS, 2) fmha_simt_async_kernel(const __grid_constant__ SimtLaunch L) {
    using C = AsyncCfg<DQKP, DVP, VT>;
    extern __shared__ __align__(16) uint8_t smb[];
    float* sQ = reinterpret_cast<float*>(smb);
    uint8_t* sKb = smb + C::Q_BYTES;                    // [2][kBK][LDQ] fp32
    uint8_t* sVb = sKb + 2 * C::K_BYTES;                // [2][kBK][LDV] VT
    float* sP = reinterpret_cast<float*>(sVb + 2 * C::V_BYTES);

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
    const int64_t Nk = L.Nk;
    const float scale = L.scale;
    const bool causal = L.causal != 0;

    load_tile(sQ, C::LDQ, DQKP, L.q, L.q_dtype, b * L.qs[0] + h * L.qs[1], L.qs[2], L.qs[3], q0, L.Nq, dqk,
              vec_ok(L.q, L.q_dtype, L.qs));
    int64_t nkb = (Nk + kBK - 1) / kBK;
    if (causal) {
        const int64_t last = (q0 + kBQ - 1 < L.Nq - 1 ? q0 + kBQ - 1 : L.Nq - 1);
        const int64_t need = last / kBK + 1;
        if (need < nkb) nkb = need;
    }
    const float* kg = static_cast<const float*>(L.k) + b * L.ks[0] + h * L.ks[1];
    const uint8_t* vg = static_cast<const uint8_t*>(L.v) + (b * L.vs[0] + h * L.vs[1]) * C::VEB;
    const int64_t ks2 = L.ks[2], vs2 = L.vs[2];
    auto issue = [&](int64_t kb) {
        const int64_t k0 = kb * kBK;
        float* dk = reinterpret_cast<float*>(sKb + (kb & 1) * C::K_BYTES);
        uint8_t* dvb = sVb + (kb & 1) * C::V_BYTES;
        constexpr int KCH = DQKP / 4;
        for (int idx = tid; idx < kBK * KCH; idx += kThreadsS) {
            const int r = idx / KCH, col = (idx - r * KCH) * 4;
            const bool ok = (k0 + r < Nk) && col < dqk;
            cp_async16(dk + r * C::LDQ + col, ok ? static_cast<const void*>(kg + (k0 + r) * ks2 + col) : L.k, ok);
        }
        constexpr int VE = 16 / C::VEB;  // elements per 16-byte chunk
        constexpr int VCH = DVP / VE;
        for (int idx = tid; idx < kBK * VCH; idx += kThreadsS) {
            const int r = idx / VCH, col = (idx - r * VCH) * VE;
            const bool ok = (k0 + r < Nk) && col < dv;
            cp_async16(dvb + (static_cast<size_t>(r) * C::LDV + col) * C::VEB,
                       ok ? static_cast<const void*>(vg + ((k0 + r) * vs2 + col) * C::VEB) : L.v, ok);
        }
    };

    float m[4], l[4], o[4][4 * C::G];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        m[r] = -INFINITY;
        l[r] = 0.f;
#pragma unroll
        for (int c = 0; c < 4 * C::G; ++c) o[r][c] = 0.f;
    }
    issue(0);
    cp_async_commit();
    for (int64_t kb = 0; kb < nkb; ++kb) {
        const int64_t k0 = kb * kBK;
        if (kb + 1 < nkb) issue(kb + 1);
        cp_async_commit();
        cp_async_wait1();  // this thread's copies of block kb have landed
        __syncthreads();   // ... and everyone else's
        const float* sK = reinterpret_cast<const float*>(sKb + (kb & 1) * C::K_BYTES);
        const uint8_t* sV = sVb + (kb & 1) * C::V_BYTES;
        float s[4][4];
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int i = 0; i < 4; ++i) s[r][i] = 0.f;
#pragma unroll 4
        for (int d = 0; d < DQKP; d += 4) {
            float4 a[4], kk[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) a[r] = *reinterpret_cast<const float4*>(sQ + (ty * 4 + r) * C::LDQ + d);
#pragma unroll
            for (int i = 0; i < 4; ++i) kk[i] = *reinterpret_cast<const float4*>(sK + (tx + 16 * i) * C::LDQ + d);
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    s[r][i] = fmaf(a[r].x, kk[i].x, s[r][i]);
                    s[r][i] = fmaf(a[r].y, kk[i].y, s[r][i]);
                    s[r][i] = fmaf(a[r].z, kk[i].z, s[r][i]);
                    s[r][i] = fmaf(a[r].w, kk[i].w, s[r][i]);
                }
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int64_t qrow = q0 + ty * 4 + r;
            float mx = -INFINITY;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int64_t kv = k0 + tx + 16 * i;
                float v = s[r][i] * scale;
                if (kv >= Nk || (causal && kv > qrow)) v = -INFINITY;
                if (L.mask.data != nullptr && kv < Nk && qrow < L.Nq) {
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
            for (int c = 0; c < 4 * C::G; ++c) o[r][c] *= alpha;
#pragma unroll
            for (int i = 0; i < 4; ++i) sP[(ty * 4 + r) * kLdP + tx + 16 * i] = s[r][i];
        }
        __syncthreads();
#pragma unroll 2
        for (int c = 0; c < kBK; c += 4) {
            float4 p[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) p[r] = *reinterpret_cast<const float4*>(sP + (ty * 4 + r) * kLdP + c);
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
#pragma unroll
                for (int g = 0; g < C::G; ++g) {
                    const float4 v = v4<VT>(sV, C::LDV, c + cc, 64 * g + 4 * tx);
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        const float pr = cc == 0 ? p[r].x : cc == 1 ? p[r].y : cc == 2 ? p[r].z : p[r].w;
                        o[r][4 * g + 0] = fmaf(pr, v.x, o[r][4 * g + 0]);
                        o[r][4 * g + 1] = fmaf(pr, v.y, o[r][4 * g + 1]);
                        o[r][4 * g + 2] = fmaf(pr, v.z, o[r][4 * g + 2]);
                        o[r][4 * g + 3] = fmaf(pr, v.w, o[r][4 * g + 3]);
                    }
                }
            }
        }
        __syncthreads();  // buffers kb & 1 and sP are free for the next block
    }
    const int64_t obase = b * L.os[0] + h * L.os[1];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const int64_t qrow = q0 + ty * 4 + r;
        if (qrow >= L.Nq) continue;
        const float inv = 1.f / l[r];
#pragma unroll
        for (int g = 0; g < C::G; ++g)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int col = 64 * g + 4 * tx + e;
                if (col < dv)
                    store_from_f32(L.out, obase + qrow * L.os[2] + col * L.os[3], L.out_dtype, o[r][4 * g + e] * inv);
            }
    }
}

template <int DQKP, int DVP, int VT>
int launch_simt_async(const SimtLaunch& L, cudaStream_t stream) {
    using C = AsyncCfg<DQKP, DVP, VT>;
    auto kern = fmha_simt_async_kernel<DQKP, DVP, VT>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(C::SMEM)) !=
        cudaSuccess)
        return ADA_ERR_LAUNCH;
    const int64_t nqb = (L.Nq + kBQ - 1) / kBQ;
    const int64_t grid = nqb * L.B * L.H;
    if (grid <= 0) return ADA_OK;
    if (grid > 0x7fffffffLL) return ADA_ERR_UNSUPPORTED;
    kern<<<static_cast<unsigned>(grid), kThreadsS, C::SMEM, stream>>>(L);
    return cudaGetLastError() == cudaSuccess ? ADA_OK : ADA_ERR_LAUNCH;
}

template <int DQKP, int DVP>
int launch_simt_async_v(const SimtLaunch& L, cudaStream_t stream) {
    if (L.v_dtype == ADA_F32) return launch_simt_async<DQKP, DVP, ADA_F32>(L, stream);
    if (L.v_dtype == ADA_F16) return launch_simt_async<DQKP, DVP, ADA_F16>(L, stream);
    return launch_simt_async<DQKP, DVP, ADA_BF16>(L, stream);
}

// K fp32 and K, V rows 16-byte aligned with widths in whole 16-byte chunks.
bool async_ok(const SimtLaunch& L) {
    auto rows16 = [](const void* p, const int64_t* st, int eb) {
        if ((reinterpret_cast<uintptr_t>(p) & 15u) != 0 || st[3] != 1) return false;
        for (int i = 0; i < 3; ++i)
            if (((st[i] * eb) % 16) != 0) return false;
        return true;
    };
    if (L.k_dtype != ADA_F32 || (L.dqk % 4) != 0 || !rows16(L.k, L.ks, 4)) return false;
    if (L.v_dtype != ADA_F32 && L.v_dtype != ADA_F16 && L.v_dtype != ADA_BF16) return false;
    const int veb = L.v_dtype == ADA_F32 ? 4 : 2;
    return (L.dv % (16 / veb)) == 0 && rows16(L.v, L.vs, veb);
}

template <int DQKP, int DVP>
int launch_simt(const SimtLaunch& L, cudaStream_t stream) {
    using C = SimtCfg<DQKP, DVP>;
    auto kern = fmha_simt_kernel<DQKP, DVP>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(C::SMEM)) !=
        cudaSuccess)
        return ADA_ERR_LAUNCH;
    const int64_t nqb = (L.Nq + kBQ - 1) / kBQ;
    const int64_t grid = nqb * L.B * L.H;
    if (grid <= 0) return ADA_OK;
    if (grid > 0x7fffffffLL) return ADA_ERR_UNSUPPORTED;
    kern<<<static_cast<unsigned>(grid), kThreadsS, C::SMEM, stream>>>(L);
    return cudaGetLastError() == cudaSuccess ? ADA_OK : ADA_ERR_LAUNCH;
}

}  // namespace

int launch_fmha_simt(const SimtLaunch& L, cudaStream_t stream) {
    if (L.dqk > 128 || L.dv > 128 || L.dqk <= 0 || L.dv <= 0) return ADA_ERR_UNSUPPORTED;
    const int qp = L.dqk <= 32 ? 32 : (L.dqk <= 64 ? 64 : 128);
    const bool v128 = L.dv > 64;
    if (qp >= 64 && async_ok(L)) {
        if (qp == 64) return v128 ? launch_simt_async_v<64, 128>(L, stream) : launch_simt_async_v<64, 64>(L, stream);
        return v128 ? launch_simt_async_v<128, 128>(L, stream) : launch_simt_async_v<128, 64>(L, stream);
    }
    if (qp == 32) return v128 ? launch_simt<32, 128>(L, stream) : launch_simt<32, 64>(L, stream);
    if (qp == 64) return v128 ? launch_simt<64, 128>(L, stream) : launch_simt<64, 64>(L, stream);
    return v128 ? launch_simt<128, 128>(L, stream) : launch_simt<128, 64>(L, stream);
}

}  // namespace ada
