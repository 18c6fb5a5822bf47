// Operand preparation for the attention kernels, driven by the per-head
// decision table on the device (no host round trip):
//   prep16  heads computed by the 16-bit tensor-core kernels that cannot be
//           read in place: cast to the compute dtype (adaattn.py:303-305,
//           :361-363), or project q and k through rank_proj_down first
//           (adaattn.py:357-358, a Linear in the inputs' dtype), and pad the
//           head dimension with zeros to a whole 128-byte row.
//   prep32  FP32 low-rank heads: q_low / k_low in fp32 for the SIMT kernel.
//   prep8   FP8 heads in E4M3 mode: per-tile amax, then tile-scaled E4M3
//           values (Q, K: one scale per 128-row tile; V: one per head).
//   split   FP32 low-rank heads of 16-bit inputs for the tensor cores:
//           q_low / k_low (already rounded to the inputs' dtype) scaled by a
//           power of two per 128-row tile, v by one per head, into fp16 --
//           exact for 16-bit values inside fp16's range after scaling.
#include "ada_common.cuh"
#include "ada_internal.h"

namespace ada {
namespace {

constexpr int kRows = 64;
constexpr int kThreads = 256;

// x[64 rows] . W^T -> y[64 rows, r] with W^T staged in shared memory as fp32.
// Each thread owns one row and r/4 output columns (col = c4 + 4*i). The
// result is rounded to the inputs' dtype, as the reference's Linear returns
// a tensor of that dtype.
struct ProjSmem {
    float* w_t;  // [D][r]
    float* x;    // [kRows][D + 1]
};

__device__ void stage_weight(const PrepLaunch& L, float* w_t) {
    const int D = static_cast<int>(L.D), r = static_cast<int>(L.r);
    for (int i = threadIdx.x; i < D * r; i += kThreads) {
        const int rr = i / D, d = i - rr * D;
        w_t[d * r + rr] = load_as_f32(L.w_down, i, L.w_dtype);
    }
}

__device__ void stage_rows(const void* x, int dtype, const int64_t* st, int64_t b, int64_t h,
                           int64_t row0, int64_t nrows, int D, float* sx) {
    const int64_t base = b * st[0] + h * st[1];
    for (int i = threadIdx.x; i < kRows * D; i += kThreads) {
        const int rr = i / D, d = i - rr * D;
        const int64_t row = row0 + rr;
        sx[rr * (D + 1) + d] = row < nrows ? load_as_f32(x, base + row * st[2] + d * st[3], dtype) : 0.f;
    }
}

// y[c] for this thread's row; cols c = c4 + 4*i, i < 32 (r <= 128).
__device__ void project_row(const float* sx, const float* w_t, int D, int r, int row, int c4,
                            float (&y)[32]) {
#pragma unroll
    for (int i = 0; i < 32; ++i) y[i] = 0.f;
    const float* xr = sx + row * (D + 1);
    for (int d = 0; d < D; ++d) {
        const float xv = xr[d];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const int c = c4 + 4 * i;
            if (c < r) y[i] = fmaf(xv, w_t[d * r + c], y[i]);
        }
    }
}

__global__ void __launch_bounds__(kThreads) prep16_kernel(const __grid_constant__ PrepLaunch L) {
    extern __shared__ float sm[];
    const int64_t bh = blockIdx.y;
    int prec, low;
    get_decision(L.dec, bh, &prec, &low);
    if (!((L.tc16_mask >> prec) & 1u)) return;
    const int cd = ((L.f16_mask >> prec) & 1u) ? ADA_F16 : ADA_BF16;
    const bool needs = low || cd != L.in_dtype || !L.direct_ok;
    if (!needs) return;
    const int64_t b = bh / L.H, h = bh % L.H;
    const int D = static_cast<int>(L.D);
    const int r = static_cast<int>(L.r);
    const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kRows;
    const int dqk_w = low ? L.dqk_low : L.dqk_dense;

    float* w_t = sm;
    float* sx = sm + (low ? D * r : 0);
    if (low) stage_weight(L, w_t);

    for (int which = 0; which < 2; ++which) {  // 0: q, 1: k
        const int64_t nrows = which == 0 ? L.Nq : L.Nk;
        if (row0 >= nrows) continue;
        const void* x = which == 0 ? L.q : L.k;
        const int64_t* st = which == 0 ? L.qs : L.ks;
        uint16_t* dst = reinterpret_cast<uint16_t*>(which == 0 ? L.ws16_q : L.ws16_k);
        const int64_t plane = (which == 0 ? L.Nq : L.Nk) * L.ld16_qk;
        if (low) {
            __syncthreads();
            stage_rows(x, L.in_dtype, st, b, h, row0, nrows, D, sx);
            __syncthreads();
            const int row = threadIdx.x >> 2, c4 = threadIdx.x & 3;
            float y[32];
            project_row(sx, w_t, D, r, row, c4, y);
            const int64_t grow = row0 + row;
            if (grow < nrows) {
                void* out = dst + bh * plane + grow * L.ld16_qk;
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const int c = c4 + 4 * i;
                    if (c < dqk_w) store_from_f32(out, c, cd, c < r ? round_to(y[i], L.in_dtype) : 0.f);
                }
            }
        } else {
            const int64_t base = b * st[0] + h * st[1];
            for (int i = threadIdx.x; i < kRows * dqk_w; i += kThreads) {
                const int rr = i / dqk_w, c = i - rr * dqk_w;
                const int64_t grow = row0 + rr;
                if (grow >= nrows) continue;
                const float val = c < D ? load_as_f32(x, base + grow * st[2] + c * st[3], L.in_dtype) : 0.f;
                store_from_f32(dst + bh * plane + grow * L.ld16_qk, c, cd, val);
            }
        }
    }
    if (row0 < L.Nk) {
        const int64_t base = b * L.vs[0] + h * L.vs[1];
        uint16_t* dst = reinterpret_cast<uint16_t*>(L.ws16_v) + bh * L.Nk * L.ld16_v;
        for (int i = threadIdx.x; i < kRows * L.dv_pad; i += kThreads) {
            const int rr = i / L.dv_pad, c = i - rr * L.dv_pad;
            const int64_t grow = row0 + rr;
            if (grow >= L.Nk) continue;
            const float val = c < D ? load_as_f32(L.v, base + grow * L.vs[2] + c * L.vs[3], L.in_dtype) : 0.f;
            store_from_f32(dst + grow * L.ld16_v, c, cd, val);
        }
    }
}

// Copy 64 rows of x [B,H,N,D] (row stride st[2]) into a 16-bit region row of
// `width` columns in dtype cd, zero padded past D; 8 elements per thread step,
// 16-byte accesses when `vec` says the source allows it.
__device__ void cast_rows(const void* x, int in_dtype, const int64_t* st, int64_t b, int64_t h, int64_t row0,
                          int64_t nrows, int D, uint16_t* dst_plane, int64_t ld, int width, int cd, bool vec) {
    const int groups = width / 8;
    const int64_t base = b * st[0] + h * st[1];
    for (int i = threadIdx.x; i < kRows * groups; i += kThreads) {
        const int rr = i / groups, g = i - rr * groups;
        const int64_t grow = row0 + rr;
        if (grow >= nrows) continue;
        const int c0 = g * 8;
        float v[8];
        if (vec && c0 + 8 <= D) {
            const int64_t e = base + grow * st[2] + c0;
            if (in_dtype == ADA_F32) {
                const float4 a = reinterpret_cast<const float4*>(x)[e / 4];
                const float4 c = reinterpret_cast<const float4*>(x)[e / 4 + 1];
                v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
                v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
            } else {
                const uint4 a = reinterpret_cast<const uint4*>(x)[e / 8];
                const uint32_t w4[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    if (in_dtype == ADA_BF16) {
                        const __nv_bfloat162 p = *reinterpret_cast<const __nv_bfloat162*>(&w4[k]);
                        v[2 * k] = __low2float(p);
                        v[2 * k + 1] = __high2float(p);
                    } else {
                        const __half2 p = *reinterpret_cast<const __half2*>(&w4[k]);
                        v[2 * k] = __low2float(p);
                        v[2 * k + 1] = __high2float(p);
                    }
                }
            }
        } else {
#pragma unroll
            for (int k = 0; k < 8; ++k)
                v[k] = (c0 + k < D) ? load_as_f32(x, base + grow * st[2] + (c0 + k) * st[3], in_dtype) : 0.f;
        }
        uint32_t p[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
            p[k] = cd == ADA_F16 ? pack_f16x2(v[2 * k], v[2 * k + 1]) : pack_bf16x2(v[2 * k], v[2 * k + 1]);
        reinterpret_cast<uint4*>(dst_plane + grow * ld)[g] = make_uint4(p[0], p[1], p[2], p[3]);
    }
}

__global__ void __launch_bounds__(kThreads) cast16_kernel(const __grid_constant__ PrepLaunch L,
                                                          int skip_low_rank_qk, int vec_q, int vec_k,
                                                          int vec_v) {
    const int64_t bh = blockIdx.y;
    int prec, low;
    get_decision(L.dec, bh, &prec, &low);
    if (!((L.tc16_mask >> prec) & 1u)) return;
    const int cd = ((L.f16_mask >> prec) & 1u) ? ADA_F16 : ADA_BF16;
    if (!(low || cd != L.in_dtype || !L.direct_ok)) return;
    const int64_t b = bh / L.H, h = bh % L.H;
    const int D = static_cast<int>(L.D);
    const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kRows;
    const bool qk_in_place = !low && L.mixed16 && cd == ADA_F16 && L.in_dtype == ADA_BF16;
    if (!(low && skip_low_rank_qk) && !qk_in_place) {
        if (row0 < L.Nq)
            cast_rows(L.q, L.in_dtype, L.qs, b, h, row0, L.Nq, D,
                      reinterpret_cast<uint16_t*>(L.ws16_q) + bh * L.Nq * L.ld16_qk, L.ld16_qk, L.dqk_dense, cd,
                      vec_q != 0);
        if (row0 < L.Nk)
            cast_rows(L.k, L.in_dtype, L.ks, b, h, row0, L.Nk, D,
                      reinterpret_cast<uint16_t*>(L.ws16_k) + bh * L.Nk * L.ld16_qk, L.ld16_qk, L.dqk_dense, cd,
                      vec_k != 0);
    }
    // v read in place by the attention kernel (converted there for FP16 heads of bf16 inputs)
    const bool v_in_place = L.v_direct && (cd == L.in_dtype || (cd == ADA_F16 && L.in_dtype == ADA_BF16));
    if (row0 < L.Nk && !v_in_place)
        cast_rows(L.v, L.in_dtype, L.vs, b, h, row0, L.Nk, D,
                  reinterpret_cast<uint16_t*>(L.ws16_v) + bh * L.Nk * L.ld16_v, L.ld16_v, L.dv_pad, cd, vec_v != 0);
}

__global__ void __launch_bounds__(kThreads) prep32_kernel(const __grid_constant__ PrepLaunch L) {
    extern __shared__ float sm[];
    const int64_t bh = blockIdx.y;
    int prec, low;
    get_decision(L.dec, bh, &prec, &low);
    if (!low || !((L.fp32_mask >> prec) & 1u)) return;
    const int64_t b = bh / L.H, h = bh % L.H;
    const int D = static_cast<int>(L.D);
    const int r = static_cast<int>(L.r);
    const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kRows;
    float* w_t = sm;
    float* sx = sm + D * r;
    stage_weight(L, w_t);
    for (int which = 0; which < 2; ++which) {
        const int64_t nrows = which == 0 ? L.Nq : L.Nk;
        if (row0 >= nrows) continue;
        __syncthreads();
        stage_rows(which == 0 ? L.q : L.k, L.in_dtype, which == 0 ? L.qs : L.ks, b, h, row0, nrows, D, sx);
        __syncthreads();
        const int row = threadIdx.x >> 2, c4 = threadIdx.x & 3;
        float y[32];
        project_row(sx, w_t, D, r, row, c4, y);
        const int64_t grow = row0 + row;
        if (grow < nrows) {
            float* out = (which == 0 ? L.ws32_q : L.ws32_k) + (bh * nrows + grow) * r;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const int c = c4 + 4 * i;
                if (c < r) out[c] = round_to(y[i], L.in_dtype);
            }
        }
    }
}

// ---------------- E4M3 ----------------
// pass 0: amax of each 128-row tile of Q (or q_low), K (or k_low) and V.
// pass 1: quantise with scale = amax / 448 (1 when amax is 0); V uses the
//         largest tile amax of its head.
__global__ void __launch_bounds__(kThreads) prep8_kernel(const __grid_constant__ PrepLaunch L, int pass) {
    extern __shared__ float sm[];
    __shared__ unsigned int s_amax[3];
    __shared__ float s_scale[3];
    const int64_t bh = blockIdx.y;
    int prec, low;
    get_decision(L.dec, bh, &prec, &low);
    if (!((L.fp8_mask >> prec) & 1u)) return;
    const int64_t b = bh / L.H, h = bh % L.H;
    const int D = static_cast<int>(L.D);
    const int r = static_cast<int>(L.r);
    const int64_t tile = blockIdx.x;
    if (threadIdx.x < 3) s_amax[threadIdx.x] = 0u;
    // low_src16: q_low/k_low already sit in the 16-bit region (written by the
    // tensor-core projection in the inputs' dtype); no projection here.
    const bool src16 = low && L.low_src16;
    float* w_t = sm;
    float* sx = sm + ((low && !src16) ? D * r : 0);
    if (low && !src16) stage_weight(L, w_t);
    if (pass == 1 && threadIdx.x == 0) {
        float sq = 1.f, sk = 1.f, svv = 0.f;
        if (tile < L.nt_q) {
            const float a = L.amax_q[bh * L.nt_q + tile];
            sq = a > 0.f ? a / 448.f : 1.f;
            L.scale_q[bh * L.nt_q + tile] = sq;
        }
        if (tile < L.nt_k) {
            const float a = L.amax_k[bh * L.nt_k + tile];
            sk = a > 0.f ? a / 448.f : 1.f;
            L.scale_k[bh * L.nt_k + tile] = sk;
        }
        for (int64_t t = 0; t < L.nt_k; ++t) svv = fmaxf(svv, L.amax_v[bh * L.nt_k + t]);
        const float sv = svv > 0.f ? svv / 448.f : 1.f;
        if (tile == 0) L.scale_v[bh] = sv;
        s_scale[0] = sq;
        s_scale[1] = sk;
        s_scale[2] = sv;
    }
    __syncthreads();
    for (int which = 0; which < 3; ++which) {  // q, k, v
        const int64_t nrows = which == 0 ? L.Nq : L.Nk;
        const int64_t nt = which == 0 ? L.nt_q : L.nt_k;
        if (tile >= nt) continue;
        const void* x = which == 0 ? L.q : (which == 1 ? L.k : L.v);
        const int64_t* st = which == 0 ? L.qs : (which == 1 ? L.ks : L.vs);
        int64_t st16[4];
        if (src16 && which < 2) {
            // [B*H][N][ld16] plane of this head, read from its own base
            x = reinterpret_cast<const uint16_t*>(which == 0 ? L.ws16_q : L.ws16_k) + bh * nrows * L.ld16_qk;
            st16[0] = 0;
            st16[1] = 0;
            st16[2] = L.ld16_qk;
            st16[3] = 1;
            st = st16;
        }
        uint8_t* dst8 = which == 0 ? L.ws8_q : (which == 1 ? L.ws8_k : L.ws8_v);
        const bool proj = low && which < 2 && !src16;
        const int width = (low && which < 2) ? r : D;
        float amax = 0.f;
        for (int half = 0; half < 2; ++half) {
            const int64_t row0 = tile * 128 + half * kRows;
            if (row0 >= nrows) break;
            __syncthreads();
            if (proj) {
                stage_rows(x, L.in_dtype, st, b, h, row0, nrows, D, sx);
                __syncthreads();
                const int row = threadIdx.x >> 2, c4 = threadIdx.x & 3;
                float y[32];
                project_row(sx, w_t, D, r, row, c4, y);
                const int64_t grow = row0 + row;
                const bool rok = grow < nrows;
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const int c = c4 + 4 * i;
                    const float val = (rok && c < r) ? round_to(y[i], L.in_dtype) : 0.f;
                    amax = fmaxf(amax, fabsf(val));
                    if (pass == 1 && rok) {
                        const float qv = val / s_scale[which];
                        dst8[(bh * nrows + grow) * 128 + c] =
                            __nv_cvt_float_to_fp8(qv, __NV_SATFINITE, __NV_E4M3);
                    }
                }
            } else {
                const int64_t base = b * st[0] + h * st[1];
                for (int i = threadIdx.x; i < kRows * 128; i += kThreads) {
                    const int rr = i >> 7, c = i & 127;
                    const int64_t grow = row0 + rr;
                    if (grow >= nrows) continue;
                    const float val = c < width ? load_as_f32(x, base + grow * st[2] + c * st[3], L.in_dtype) : 0.f;
                    amax = fmaxf(amax, fabsf(val));
                    if (pass == 1) {
                        dst8[(bh * nrows + grow) * 128 + c] =
                            __nv_cvt_float_to_fp8(val / s_scale[which], __NV_SATFINITE, __NV_E4M3);
                    }
                }
            }
        }
        if (pass == 0) {
            for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            if ((threadIdx.x & 31) == 0) atomicMax(&s_amax[which], __float_as_uint(amax));
        }
    }
    if (pass == 0) {
        __syncthreads();
        if (threadIdx.x == 0) {
            if (tile < L.nt_q) L.amax_q[bh * L.nt_q + tile] = __uint_as_float(s_amax[0]);
            if (tile < L.nt_k) {
                L.amax_k[bh * L.nt_k + tile] = __uint_as_float(s_amax[1]);
                L.amax_v[bh * L.nt_k + tile] = __uint_as_float(s_amax[2]);
            }
        }
    }
}

size_t proj_smem(const PrepLaunch& L, bool with_weight) {
    size_t f = static_cast<size_t>(kRows) * (L.D + 1);
    if (with_weight) f += static_cast<size_t>(L.D) * L.r;
    return f * sizeof(float);
}

template <typename K>
int set_smem(K kern, size_t smem) {
    if (smem > 48 * 1024)
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
            cudaSuccess)
            return ADA_ERR_LAUNCH;
    return ADA_OK;
}

}  // namespace

int launch_prep16(const PrepLaunch& L, cudaStream_t stream) {
    const int64_t nt = ((L.Nq > L.Nk ? L.Nq : L.Nk) + kRows - 1) / kRows;
    if (nt == 0 || L.B * L.H == 0) return ADA_OK;
    const size_t smem = proj_smem(L, L.w_down != nullptr);
    if (set_smem(prep16_kernel, smem) != ADA_OK) return ADA_ERR_LAUNCH;
    prep16_kernel<<<dim3(static_cast<unsigned>(nt), static_cast<unsigned>(L.B * L.H)), kThreads, smem, stream>>>(L);
    return cudaGetLastError() == cudaSuccess ? ADA_OK : ADA_ERR_LAUNCH;
}

// Power of two s with max|x| / s < 2^15: the scaled values and their fp16
// high parts stay below fp16's largest finite value (65504).
__device__ __forceinline__ float split_scale(float amax) {
    if (!(amax > 0.f) || !(amax < INFINITY)) return 1.f;
    int e;
    frexpf(amax, &e);  // amax = m * 2^e, m in [0.5, 1)
    return ldexpf(1.f, e - 15 < -126 ? -126 : e - 15);
}

__device__ __forceinline__ float block_max256(float v, float* red) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float m = red[0];
#pragma unroll
    for (int i = 1; i < kThreads / 32; ++i) m = fmaxf(m, red[i]);
    return m;
}

// 0: not served; 1: low-rank head; 2: dense head.
__device__ __forceinline__ int split_head(const PrepLaunch& L, int64_t bh) {
    int prec, low;
    get_decision(L.dec, bh, &prec, &low);
    if (!((L.split_mask >> prec) & 1u)) return 0;
    if (low) return L.split_low ? 1 : 0;
    return L.split_dense ? 2 : 0;
}

// max |v| of one 128-row tile of a selected head, folded into amax_v[bh].
__global__ void __launch_bounds__(kThreads) split_vamax_kernel(const __grid_constant__ PrepLaunch L, int vec_v) {
    __shared__ float red[kThreads / 32];
    const int64_t bh = blockIdx.y;
    if (split_head(L, bh) == 0) return;
    const int64_t b = bh / L.H, h = bh % L.H;
    const int D = static_cast<int>(L.D);
    const int groups = (D + 7) / 8;
    const int64_t row0 = static_cast<int64_t>(blockIdx.x) * 128;
    const int rows = static_cast<int>((L.Nk - row0) < 128 ? (L.Nk - row0) : 128);
    const int64_t base = b * L.vs[0] + h * L.vs[1];
    float a = 0.f;
    for (int i = threadIdx.x; i < rows * groups; i += kThreads) {
        const int rr = i / groups, g = i - rr * groups;
        float v[8];
        load8(L.v, L.in_dtype, base + (row0 + rr) * L.vs[2], L.vs[3], g * 8, D, vec_v != 0, v);
#pragma unroll
        for (int k = 0; k < 8; ++k) a = fmaxf(a, fabsf(v[k]));
    }
    a = block_max256(a, red);
    if (threadIdx.x == 0) atomicMax(L.split_amax_v + bh, __float_as_uint(a));  // a >= 0: bits order as values
}

__device__ __forceinline__ uint4 pack8_f16(const float (&v)[8], float inv) {
    return make_uint4(pack_f16x2(v[0] * inv, v[1] * inv), pack_f16x2(v[2] * inv, v[3] * inv),
                      pack_f16x2(v[4] * inv, v[5] * inv), pack_f16x2(v[6] * inv, v[7] * inv));
}

// One 128-row tile of q (or q_low), k (or k_low) and v of a selected head.
// vec_*: the source's rows allow 16-byte loads.
__global__ void __launch_bounds__(kThreads) split_kernel(const __grid_constant__ PrepLaunch L, int vec_q, int vec_k,
                                                         int vec_v) {
    __shared__ float red[kThreads / 32];
    const int64_t bh = blockIdx.y;
    const int kind = split_head(L, bh);
    if (kind == 0) return;
    const int64_t b = bh / L.H, h = bh % L.H;
    const int64_t tile = blockIdx.x;
    // low rank: fp32 q_low/k_low [B*H][N][r] -> 64 columns;
    // dense: the 16-bit inputs (any strides) -> dqk_dense columns
    const int width = kind == 1 ? static_cast<int>(L.r) : static_cast<int>(L.D);
    const int wout = kind == 1 ? 64 : L.dqk_dense;
    const int groups = wout / 8;
    const bool scale_qk = kind == 1 ? L.split_qk_low != 0 : L.split_qk_dense != 0;
    for (int which = 0; which < (scale_qk ? 2 : 0); ++which) {
        const int64_t N = which == 0 ? L.Nq : L.Nk;
        const int64_t nt = which == 0 ? L.nt_q : L.nt_k;
        if (tile >= nt) continue;
        const int64_t row0 = tile * 128;
        const int rows = static_cast<int>((N - row0) < 128 ? (N - row0) : 128);
        const void* src;
        int dt;
        int64_t base, rs, cs;
        bool vec;
        if (kind == 1) {
            src = which == 0 ? L.ws32_q : L.ws32_k;
            dt = ADA_F32;
            base = (bh * N + row0) * width;
            rs = width;
            cs = 1;
            vec = (width % 4) == 0;
        } else {
            const int64_t* st = which == 0 ? L.qs : L.ks;
            src = which == 0 ? L.q : L.k;
            dt = L.in_dtype;
            base = b * st[0] + h * st[1] + row0 * st[2];
            rs = st[2];
            cs = st[3];
            vec = (which == 0 ? vec_q : vec_k) != 0;
        }
        // at most 128 rows x 16 groups = 8 groups per thread, held in registers
        float x[8][8];
        float a = 0.f;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = threadIdx.x + u * kThreads;
            if (i < rows * groups) {
                const int rr = i / groups, g = i - rr * groups;
                load8(src, dt, base + rr * rs, cs, g * 8, width, vec, x[u]);
#pragma unroll
                for (int k = 0; k < 8; ++k) a = fmaxf(a, fabsf(x[u][k]));
            }
        }
        const float sc = split_scale(block_max256(a, red));
        if (threadIdx.x == 0) (which == 0 ? L.split_sq : L.split_sk)[bh * nt + tile] = sc;
        const float inv = 1.f / sc;  // a power of two: exact
        uint16_t* dst = (which == 0 ? L.wss_q : L.wss_k) + (bh * N + row0) * L.split_ld;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = threadIdx.x + u * kThreads;
            if (i < rows * groups) {
                const int rr = i / groups, g = i - rr * groups;
                reinterpret_cast<uint4*>(dst + rr * L.split_ld)[g] = pack8_f16(x[u], inv);
            }
        }
    }
    if (tile < L.nt_k) {
        const float sv = split_scale(__uint_as_float(L.split_amax_v[bh]));
        if (tile == 0 && threadIdx.x == 0) L.split_sv[bh] = sv;
        const float inv = 1.f / sv;
        const int D = static_cast<int>(L.D);
        const int64_t row0 = tile * 128;
        const int rows = static_cast<int>((L.Nk - row0) < 128 ? (L.Nk - row0) : 128);
        const int64_t base = b * L.vs[0] + h * L.vs[1];
        uint16_t* dst = L.wss_v + (bh * L.Nk + row0) * 128;
        for (int i = threadIdx.x; i < rows * 16; i += kThreads) {
            const int rr = i >> 4, g = i & 15;
            float v[8];
            load8(L.v, L.in_dtype, base + (row0 + rr) * L.vs[2], L.vs[3], g * 8, D, vec_v != 0, v);
            reinterpret_cast<uint4*>(dst + rr * 128)[g] = pack8_f16(v, inv);
        }
    }
}

// E4M3 heads whose q, k need no projection here (dense heads, or low-rank
// heads whose q_low / k_low the tensor-core projection already wrote to the
// 16-bit region): pass 0 takes each V tile's amax; pass 1 quantises q and k
// with one scale per 128-row tile (the tile held in registers between its
// amax and its stores) and v with the head's scale. Same arithmetic as
// prep8: scale = amax / 448, e4m3(x / scale) saturating.
__global__ void __launch_bounds__(kThreads) quant8_kernel(const __grid_constant__ PrepLaunch L, int pass, int vec_q,
                                                          int vec_k, int vec_v) {
    __shared__ float red[kThreads / 32];
    const int64_t bh = blockIdx.y;
    int prec, low;
    get_decision(L.dec, bh, &prec, &low);
    if (!((L.fp8_mask >> prec) & 1u)) return;
    const int64_t b = bh / L.H, h = bh % L.H;
    const int D = static_cast<int>(L.D);
    const int64_t tile = blockIdx.x;
    if (pass == 0) {
        if (tile >= L.nt_k) return;
        const int64_t row0 = tile * 128;
        const int rows = static_cast<int>((L.Nk - row0) < 128 ? (L.Nk - row0) : 128);
        const int64_t base = b * L.vs[0] + h * L.vs[1];
        // all eight 16-byte loads of a thread in flight before the first use
        float x[8][8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = threadIdx.x + u * kThreads;
            if (i < rows * 16)
                load8(L.v, L.in_dtype, base + (row0 + (i >> 4)) * L.vs[2], L.vs[3], (i & 15) * 8, D,
                      vec_v != 0, x[u]);
        }
        float a = 0.f;
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (threadIdx.x + u * kThreads < rows * 16)
#pragma unroll
                for (int k = 0; k < 8; ++k) a = fmaxf(a, fabsf(x[u][k]));
        a = block_max256(a, red);
        if (threadIdx.x == 0) L.amax_v[bh * L.nt_k + tile] = a;
        return;
    }
    // pass 1: blockIdx.z picks the tensor (0 q, 1 k, 2 v), so the three
    // tiles of one (b, h, tile) stream in parallel CTAs.
    const int width = low ? static_cast<int>(L.r) : D;
    const int which = static_cast<int>(blockIdx.z);
    if (which < 2) {
        const int64_t N = which == 0 ? L.Nq : L.Nk;
        const int64_t nt = which == 0 ? L.nt_q : L.nt_k;
        if (tile >= nt) return;
        const int64_t row0 = tile * 128;
        const int rows = static_cast<int>((N - row0) < 128 ? (N - row0) : 128);
        const void* src;
        int64_t base, rs, cs;
        bool vec;
        if (low) {
            src = which == 0 ? L.ws16_q : L.ws16_k;
            base = (bh * N + row0) * L.ld16_qk;
            rs = L.ld16_qk;
            cs = 1;
            vec = true;
        } else {
            const int64_t* st = which == 0 ? L.qs : L.ks;
            src = which == 0 ? L.q : L.k;
            base = b * st[0] + h * st[1] + row0 * st[2];
            rs = st[2];
            cs = st[3];
            vec = (which == 0 ? vec_q : vec_k) != 0;
        }
        float x[8][8];
        float a = 0.f;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = threadIdx.x + u * kThreads;
            if (i < rows * 16) {
                const int rr = i >> 4, g = i & 15;
                load8(src, L.in_dtype, base + rr * rs, cs, g * 8, width, vec, x[u]);
#pragma unroll
                for (int k = 0; k < 8; ++k) a = fmaxf(a, fabsf(x[u][k]));
            }
        }
        a = block_max256(a, red);
        const float sc = a > 0.f ? a / 448.f : 1.f;
        if (threadIdx.x == 0) {
            (which == 0 ? L.amax_q : L.amax_k)[bh * nt + tile] = a;
            (which == 0 ? L.scale_q : L.scale_k)[bh * nt + tile] = sc;
        }
        uint8_t* dst = (which == 0 ? L.ws8_q : L.ws8_k) + (bh * N + row0) * 128;
        const float isc = 1.f / sc;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = threadIdx.x + u * kThreads;
            if (i < rows * 16) {
                const int rr = i >> 4, g = i & 15;
                const float* y = x[u];
                reinterpret_cast<uint2*>(dst + rr * 128)[g] = make_uint2(
                    pack_e4m3x4(div_by(y[0], sc, isc), div_by(y[1], sc, isc), div_by(y[2], sc, isc),
                                div_by(y[3], sc, isc)),
                    pack_e4m3x4(div_by(y[4], sc, isc), div_by(y[5], sc, isc), div_by(y[6], sc, isc),
                                div_by(y[7], sc, isc)));
            }
        }
    }
    if (which == 2 && tile < L.nt_k) {
        float svv = 0.f;
        for (int64_t t = 0; t < L.nt_k; ++t) svv = fmaxf(svv, L.amax_v[bh * L.nt_k + t]);
        const float sv = svv > 0.f ? svv / 448.f : 1.f;
        if (tile == 0 && threadIdx.x == 0) L.scale_v[bh] = sv;
        const int64_t row0 = tile * 128;
        const int rows = static_cast<int>((L.Nk - row0) < 128 ? (L.Nk - row0) : 128);
        const int64_t base = b * L.vs[0] + h * L.vs[1];
        uint8_t* dst = L.ws8_v + (bh * L.Nk + row0) * 128;
        const float isv = 1.f / sv;
        float x[8][8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = threadIdx.x + u * kThreads;
            if (i < rows * 16)
                load8(L.v, L.in_dtype, base + (row0 + (i >> 4)) * L.vs[2], L.vs[3], (i & 15) * 8, D,
                      vec_v != 0, x[u]);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = threadIdx.x + u * kThreads;
            if (i < rows * 16) {
                const float* y = x[u];
                reinterpret_cast<uint2*>(dst + (i >> 4) * 128)[i & 15] = make_uint2(
                    pack_e4m3x4(div_by(y[0], sv, isv), div_by(y[1], sv, isv), div_by(y[2], sv, isv),
                                div_by(y[3], sv, isv)),
                    pack_e4m3x4(div_by(y[4], sv, isv), div_by(y[5], sv, isv), div_by(y[6], sv, isv),
                                div_by(y[7], sv, isv)));
            }
        }
    }
}


// The same quantisation with each 128-row tile staged in shared memory by
// bulk async copies (one per row, issued by the row's thread), for 16-bit
// inputs whose rows are 16-byte aligned. A CTA holds one tile of one tensor
// (blockIdx.z: 0 q, 1 k, 2 v in pass 1; v in pass 0), so CTAs stay small and
// many tiles stream from HBM at once. Pass 0: V tile amax; pass 1: q / k tile
// amax and quantisation, v with the head's scale (max of the V tile amaxes).
constexpr int kStageThreads = 128;

__global__ void __launch_bounds__(kStageThreads) quant8_stage_kernel(const __grid_constant__ PrepLaunch L,
                                                                     int pass) {
    __shared__ __align__(128) uint16_t tile_s[128 * 128];
    __shared__ __align__(8) uint64_t bar;
    __shared__ float red[kStageThreads / 32];
    __shared__ int abort_flag;
    const int64_t bh = blockIdx.y;
    int prec, low;
    get_decision(L.dec, bh, &prec, &low);
    if (!((L.fp8_mask >> prec) & 1u)) return;
    const int which = pass == 0 ? 2 : static_cast<int>(blockIdx.z);
    const int64_t N = which == 0 ? L.Nq : L.Nk;
    const int64_t nt = which == 0 ? L.nt_q : L.nt_k;
    const int64_t tile = blockIdx.x;
    if (tile >= nt) return;
    const int64_t b = bh / L.H, h = bh % L.H;
    const int width = (which < 2 && low) ? static_cast<int>(L.r) : static_cast<int>(L.D);
    const int64_t row0 = tile * 128;
    const int rows = static_cast<int>((N - row0) < 128 ? (N - row0) : 128);
    const uint16_t* src;
    int64_t rs;
    if (which < 2 && low) {
        src = static_cast<const uint16_t*>(which == 0 ? L.ws16_q : L.ws16_k) + (bh * N + row0) * L.ld16_qk;
        rs = L.ld16_qk;
    } else {
        const int64_t* st = which == 0 ? L.qs : (which == 1 ? L.ks : L.vs);
        src = static_cast<const uint16_t*>(which == 0 ? L.q : (which == 1 ? L.k : L.v)) + b * st[0] +
              h * st[1] + row0 * st[2];
        rs = st[2];
    }
    const int tid = threadIdx.x;
    const uint32_t row_bytes = static_cast<uint32_t>(width) * 2u;
    if (tid == 0) {
        mbar_init(smem_u32(&bar), 1);
        abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) mbar_arrive_expect_tx(smem_u32(&bar), row_bytes * static_cast<uint32_t>(rows));
    __syncthreads();
    if (tid < rows) bulk_load(smem_u32(tile_s + tid * 128), src + tid * rs, row_bytes, smem_u32(&bar));
    const bool ok = mbar_wait(smem_u32(&bar), 0, &abort_flag, L.timeout_ns, L.status);
    // Thread t owns 16-byte chunk (t & 15) of rows t/16, t/16 + 8, ...
    const int g = tid & 15;
    const int c0 = g * 8;
    float a = 0.f;
    const bool need_amax = pass == 0 || which != 2;  // pass 1 quantises v with the head's scale
    if (ok && need_amax) {
        for (int rr = tid >> 4; rr < rows; rr += kStageThreads / 16) {
            if (c0 < width) {
                const uint4 w4 = *reinterpret_cast<const uint4*>(tile_s + rr * 128 + c0);
                const uint32_t ws[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    float x0, x1;
                    if (L.in_dtype == ADA_BF16) {
                        x0 = __uint_as_float(ws[k] << 16);
                        x1 = __uint_as_float(ws[k] & 0xffff0000u);
                    } else {
                        unpack_f16x2(ws[k], x0, x1);
                    }
                    if (c0 + 2 * k < width) a = fmaxf(a, fabsf(x0));
                    if (c0 + 2 * k + 1 < width) a = fmaxf(a, fabsf(x1));
                }
            }
        }
    }
    for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    if ((tid & 31) == 0) red[tid >> 5] = a;
    __syncthreads();
    a = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    if (pass == 0) {
        if (tid == 0) L.amax_v[bh * L.nt_k + tile] = a;
        return;
    }
    float sc;
    if (which < 2) {
        sc = a > 0.f ? a / 448.f : 1.f;
        if (tid == 0) {
            (which == 0 ? L.amax_q : L.amax_k)[bh * nt + tile] = a;
            (which == 0 ? L.scale_q : L.scale_k)[bh * nt + tile] = sc;
        }
    } else {
        float svv = 0.f;
        for (int64_t t = 0; t < L.nt_k; ++t) svv = fmaxf(svv, L.amax_v[bh * L.nt_k + t]);
        sc = svv > 0.f ? svv / 448.f : 1.f;
        if (tile == 0 && tid == 0) L.scale_v[bh] = sc;
    }
    if (!ok) return;
    const float isc = 1.f / sc;
    uint8_t* dst = (which == 0 ? L.ws8_q : (which == 1 ? L.ws8_k : L.ws8_v)) + (bh * N + row0) * 128;
    for (int rr = tid >> 4; rr < rows; rr += kStageThreads / 16) {
        float y[8];
        if (c0 < width) {
            const uint4 w4 = *reinterpret_cast<const uint4*>(tile_s + rr * 128 + c0);
            const uint32_t ws[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                if (L.in_dtype == ADA_BF16) {
                    y[2 * k] = __uint_as_float(ws[k] << 16);
                    y[2 * k + 1] = __uint_as_float(ws[k] & 0xffff0000u);
                } else {
                    unpack_f16x2(ws[k], y[2 * k], y[2 * k + 1]);
                }
            }
#pragma unroll
            for (int k = 0; k < 8; ++k)
                if (c0 + k >= width) y[k] = 0.f;
        } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) y[k] = 0.f;
        }
        reinterpret_cast<uint2*>(dst + rr * 128)[g] = make_uint2(
            pack_e4m3x4(div_by(y[0], sc, isc), div_by(y[1], sc, isc), div_by(y[2], sc, isc), div_by(y[3], sc, isc)),
            pack_e4m3x4(div_by(y[4], sc, isc), div_by(y[5], sc, isc), div_by(y[6], sc, isc), div_by(y[7], sc, isc)));
    }
}

int launch_cast16(const PrepLaunch& L, int skip_low_rank_qk, cudaStream_t stream) {
    const int64_t nt = ((L.Nq > L.Nk ? L.Nq : L.Nk) + kRows - 1) / kRows;
    if (nt == 0 || L.B * L.H == 0) return ADA_OK;
    const int eb = L.in_dtype == ADA_F32 ? 4 : 2;
    auto vec_ok = [&](const void* p, const int64_t* st) {
        if (st[3] != 1 || (L.D % 8) != 0) return 0;
        if ((reinterpret_cast<uintptr_t>(p) & 15u) != 0) return 0;
        for (int i = 0; i < 3; ++i)
            if (((st[i] * eb) % 16) != 0) return 0;
        return 1;
    };
    cast16_kernel<<<dim3(static_cast<unsigned>(nt), static_cast<unsigned>(L.B * L.H)), kThreads, 0, stream>>>(
        L, skip_low_rank_qk, vec_ok(L.q, L.qs), vec_ok(L.k, L.ks), vec_ok(L.v, L.vs));
    return cudaGetLastError() == cudaSuccess ? ADA_OK : ADA_ERR_LAUNCH;
}

int launch_prep32(const PrepLaunch& L, cudaStream_t stream) {
    const int64_t nt = ((L.Nq > L.Nk ? L.Nq : L.Nk) + kRows - 1) / kRows;
    if (nt == 0 || L.B * L.H == 0 || L.w_down == nullptr) return ADA_OK;
    const size_t smem = proj_smem(L, true);
    if (set_smem(prep32_kernel, smem) != ADA_OK) return ADA_ERR_LAUNCH;
    prep32_kernel<<<dim3(static_cast<unsigned>(nt), static_cast<unsigned>(L.B * L.H)), kThreads, smem, stream>>>(L);
    return cudaGetLastError() == cudaSuccess ? ADA_OK : ADA_ERR_LAUNCH;
}

int launch_split(const PrepLaunch& L, cudaStream_t stream) {
    const int64_t nt = L.nt_q > L.nt_k ? L.nt_q : L.nt_k;
    if (nt == 0 || L.B * L.H == 0) return ADA_OK;
    const int eb = L.in_dtype == ADA_F32 ? 4 : 2;
    auto vec_ok = [&](const void* p, const int64_t* st) {
        if (st[3] != 1 || (reinterpret_cast<uintptr_t>(p) & 15u) != 0) return 0;
        for (int i = 0; i < 3; ++i)
            if (((st[i] * eb) % 16) != 0) return 0;
        return 1;
    };
    const int vv = vec_ok(L.v, L.vs);
    if (L.nt_k > 0) {
        split_vamax_kernel<<<dim3(static_cast<unsigned>(L.nt_k), static_cast<unsigned>(L.B * L.H)), kThreads, 0,
                             stream>>>(L, vv);
        if (cudaGetLastError() != cudaSuccess) return ADA_ERR_LAUNCH;
    }
    split_kernel<<<dim3(static_cast<unsigned>(nt), static_cast<unsigned>(L.B * L.H)), kThreads, 0, stream>>>(
        L, vec_ok(L.q, L.qs), vec_ok(L.k, L.ks), vv);
    return cudaGetLastError() == cudaSuccess ? ADA_OK : ADA_ERR_LAUNCH;
}

int launch_prep8(const PrepLaunch& L, cudaStream_t stream) {
    const int64_t nt = L.nt_q > L.nt_k ? L.nt_q : L.nt_k;
    if (nt == 0 || L.B * L.H == 0) return ADA_OK;
    if (L.w_down == nullptr || L.low_src16) {
        const int eb = L.in_dtype == ADA_F32 ? 4 : 2;
        auto vec_ok = [&](const void* p, const int64_t* st) {
            if (st[3] != 1 || (reinterpret_cast<uintptr_t>(p) & 15u) != 0) return 0;
            for (int i = 0; i < 3; ++i)
                if (((st[i] * eb) % 16) != 0) return 0;
            return 1;
        };
        const dim3 grid(static_cast<unsigned>(nt), static_cast<unsigned>(L.B * L.H));
        const int vq = vec_ok(L.q, L.qs), vk = vec_ok(L.k, L.ks), vv = vec_ok(L.v, L.vs);
        // Staged path: 16-bit inputs, rows of whole 16-byte chunks, every row
        // start 16-byte aligned (the low-rank 16-bit region always is).
        const bool in16 = L.in_dtype == ADA_F16 || L.in_dtype == ADA_BF16;
        const bool rows_ok = (L.D % 8) == 0 && L.D <= 128 && vq && vk && vv &&
                             (L.w_down == nullptr || (L.r % 8) == 0);
        if (in16 && rows_ok && L.status != nullptr) {
            quant8_stage_kernel<<<grid, kStageThreads, 0, stream>>>(L, 0);
            if (cudaGetLastError() != cudaSuccess) return ADA_ERR_LAUNCH;
            quant8_stage_kernel<<<dim3(grid.x, grid.y, 3), kStageThreads, 0, stream>>>(L, 1);
            return cudaGetLastError() == cudaSuccess ? ADA_OK : ADA_ERR_LAUNCH;
        }
        quant8_kernel<<<grid, kThreads, 0, stream>>>(L, 0, vq, vk, vv);
        if (cudaGetLastError() != cudaSuccess) return ADA_ERR_LAUNCH;
        quant8_kernel<<<dim3(grid.x, grid.y, 3), kThreads, 0, stream>>>(L, 1, vq, vk, vv);
        return cudaGetLastError() == cudaSuccess ? ADA_OK : ADA_ERR_LAUNCH;
    }
    const size_t smem = proj_smem(L, L.w_down != nullptr && !L.low_src16);
    if (set_smem(prep8_kernel, smem) != ADA_OK) return ADA_ERR_LAUNCH;
    const dim3 grid(static_cast<unsigned>(nt), static_cast<unsigned>(L.B * L.H));
    prep8_kernel<<<grid, kThreads, smem, stream>>>(L, 0);
    if (cudaGetLastError() != cudaSuccess) return ADA_ERR_LAUNCH;
    prep8_kernel<<<grid, kThreads, smem, stream>>>(L, 1);
    return cudaGetLastError() == cudaSuccess ? ADA_OK : ADA_ERR_LAUNCH;
}

}  // namespace ada
