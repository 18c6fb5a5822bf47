// Randomized truncated SVD of a batch of fp32 matrices, A ~= U diag(S) Vh:
// adaattn.linalg.low_rank.randomized_svd (src/adaattn/linalg/low_rank.py:56-109)
// with the Gaussian sketch passed in.
//
//   Y   = A Omega                              panel GEMM (tensor cores)
//   repeat n_power:  Z = A^T Y,  Y = A Z       panel GEMMs          (:89-90)
//   Q   = orth(Y)                              CholeskyQR2          (:93)
//   B   = Q^T A                                panel GEMM           (:96)
//   B B^T = W diag(S^2) W^T                    Jacobi in fp64       (:99)
//   U   = Q W[:, :r],  Vh = diag(1/S) W^T B    panel applies        (:102-107)
//
// Tall-skinny operands live transposed as "panels" [k, L] (row c holds
// column c of the matrix), so every tensor-core operand of the panel GEMM is
// read K-major except A itself in A^T Y, which is read MN-major. The GEMMs
// run on tcgen05 kind::tf32 with each fp32 operand split into a tf32 head
// and an fp32 tail (three products: tail*head + head*tail + head*head); each
// 32-wide K chunk is accumulated on its own in TMEM and the chunk sums are
// added in registers, which keeps the result within a few fp32 ulps. The
// Gram matrices, the Cholesky factorisations and the eigen-solve are fp64.
//
// CholeskyQR replaces the reference's Householder QR. Both give an
// orthonormal basis of range(Y); a column whose Gram-Schmidt residual is
// below 1e-7 of its norm (numerically inside the span of the earlier
// columns) becomes a zero column of Q instead of an arbitrary completion.
// The second pass restores orthogonality lost to the conditioning of Y.
#include "ada_common.cuh"
#include "ada_internal.h"

#include <cstdio>
#include <cstring>

namespace ada {
namespace {

constexpr int kMaxSketch = 112;  // k limit: two fp64 k x k matrices in shared memory

// ---------------------------------------------------------------------------
// Panel GEMM: out^T = (A X)^T or (A^T Y)^T for one 128-row tile of out.
// ---------------------------------------------------------------------------
constexpr int kPgThreads = 256;
constexpr int kPgStages = 3;
constexpr int kPgHalf = 16384;              // one 16 KB operand buffer
constexpr int kPgStageBytes = 4 * kPgHalf;  // A head, A tail, panel head, panel tail

struct __align__(8) PgBarriers {
    uint64_t full[kPgStages];
    uint64_t split[kPgStages];
    uint64_t empty[kPgStages];
    uint64_t acc_full[2];
    uint64_t acc_empty[2];
    uint32_t tmem_base;
    int abort_flag;
};

struct PanelGemm {
    CUtensorMap ta;  // A [batch, m, n] fp32, dims {n, m, batch}; box {32,128} (NN) or {32,32} (TN)
    CUtensorMap tp;  // input panel [batch, k, L_in] fp32, dims {L_in, k, batch}; box {32, kp}
    float* out;      // output panel [batch, k, ld_out]
    int64_t out_bs, ld_out;
    int rows;  // output rows: m (NN) or n (TN)
    int kdim;  // reduction extent: n (NN) or m (TN)
    int k, kp;
    int trans;  // 0: out = (A X)^T; 1: out = (A^T Y)^T
    int batch, tiles;     // work items: (batch, 128-row tile, K split)
    int splits, cps;      // K splits per tile, 32-wide chunks per split
    unsigned int* status;
    uint64_t timeout_ns;
};

// Work item it -> (b, tile, split) and its chunk range [c0, c1).
struct PgItem {
    int b, row0, c0, c1;
};
__device__ __forceinline__ PgItem pg_item(const PanelGemm& G, int it) {
    PgItem w;
    const int split = it % G.splits;
    const int bt = it / G.splits;
    w.b = bt / G.tiles;
    w.row0 = (bt % G.tiles) * 128;
    const int nchunks = (G.kdim + 31) / 32;
    w.c0 = split * G.cps;
    w.c1 = min(nchunks, w.c0 + G.cps);
    return w;
}

__device__ __forceinline__ void split_tf32(float4& v, float4& lo) {
    float h[4] = {v.x, v.y, v.z, v.w}, l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        uint32_t t;
        asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(t) : "f"(h[i]));
        const float hh = __uint_as_float(t);
        l[i] = h[i] - hh;
        h[i] = hh;
    }
    v = make_float4(h[0], h[1], h[2], h[3]);
    lo = make_float4(l[0], l[1], l[2], l[3]);
}

// MN-major 32-bit operand (A^T in A^T Y): 128-byte rows in the 32-byte-atom
// 128B swizzle (what TMA's SWIZZLE_128B_ATOM_32B writes), 32-element MN atoms
// 4 KB apart, 4-row K groups 512 bytes apart.
__device__ __forceinline__ uint64_t make_sdesc_mn32(uint32_t saddr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(4096u >> 4) << 16;  // leading byte offset: next MN atom
    d |= static_cast<uint64_t>(512u >> 4) << 32;   // stride byte offset: next 4-row K group
    d |= static_cast<uint64_t>(1) << 46;           // descriptor version for sm_100
    d |= static_cast<uint64_t>(1) << 61;           // SWIZZLE_128B with 32-byte atoms
    return d;
}

// Accumulation: the tensor core's fp32 accumulator drifts toward zero over
// long chains of adds, so every 32-wide K chunk is summed on its own in one
// of two TMEM buffers (head*head products apart from the tail terms) and the
// chunk sums are added in registers with round-to-nearest fp32 adds.
template <int KP>
__device__ __forceinline__ void pg_split_stage(uint8_t* stage, int t) {
    float4* a = reinterpret_cast<float4*>(stage);
    float4* alo = a + kPgHalf / 16;
    for (int i = t; i < kPgHalf / 16; i += 128) {
        float4 v = a[i], lo;
        split_tf32(v, lo);
        a[i] = v;
        alo[i] = lo;
    }
    float4* p = a + 2 * (kPgHalf / 16);
    float4* plo = a + 3 * (kPgHalf / 16);
    for (int i = t; i < KP * 8; i += 128) {
        float4 v = p[i], lo;
        split_tf32(v, lo);
        p[i] = v;
        plo[i] = lo;
    }
    fence_proxy_async_smem();
}

// Persistent CTAs walk the work items with a static stride; the TMA / MMA /
// split pipeline runs across item boundaries. With several K splits per
// tile the item's partial result is added to the zeroed output with fp32
// atomics (round-to-nearest, order-dependent in the last bit).
template <int KP>
__global__ void __launch_bounds__(kPgThreads, 1) panel_gemm_kernel(const __grid_constant__ PanelGemm G) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    PgBarriers* bars = reinterpret_cast<PgBarriers*>(base + kPgStages * kPgStageBytes);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_items = G.batch * G.tiles * G.splits;
    constexpr uint32_t P_BYTES = KP * 128u;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kPgStages; ++s) {
            mbar_init(smem_u32(&bars->full[s]), 1);
            mbar_init(smem_u32(&bars->split[s]), 128);
            mbar_init(smem_u32(&bars->empty[s]), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(smem_u32(&bars->acc_full[a]), 1);
            mbar_init(smem_u32(&bars->acc_empty[a]), 128);
        }
        bars->abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(&bars->tmem_base), 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;  // buffer a: head at a*256, tail at a*256 + 128
    volatile int* abort_flag = &bars->abort_flag;
    const uint64_t tmo = G.timeout_ns;

    if (warp == 0) {
        if (lane == 0) {
            tma_prefetch_desc(&G.ta);
            tma_prefetch_desc(&G.tp);
            int g = 0;
            bool ok = true;
            for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x) {
                const PgItem w = pg_item(G, it);
                for (int c = w.c0; c < w.c1; ++c, ++g) {
                    const int st = g % kPgStages;
                    const uint32_t ph = (g / kPgStages) & 1u;
                    ok = mbar_wait(smem_u32(&bars->empty[st]), ph ^ 1u, abort_flag, tmo, G.status);
                    if (!ok) break;
                    const uint32_t fb = smem_u32(&bars->full[st]);
                    mbar_arrive_expect_tx(fb, kPgHalf + P_BYTES);
                    uint8_t* sa = base + st * kPgStageBytes;
                    if (!G.trans) {
                        tma_load_3d(smem_u32(sa), &G.ta, fb, c * 32, w.row0, w.b);
                    } else {
#pragma unroll
                        for (int q = 0; q < 4; ++q)
                            tma_load_3d(smem_u32(sa + q * 4096), &G.ta, fb, w.row0 + 32 * q, c * 32, w.b);
                    }
                    tma_load_3d(smem_u32(sa + 2 * kPgHalf), &G.tp, fb, c * 32, 0, w.b);
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = make_idesc(2, 2, G.trans ? 1u : 0u, 0, 128, KP);
            int g = 0;
            bool ok = true;
            for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x) {
                const PgItem w = pg_item(G, it);
                for (int c = w.c0; c < w.c1; ++c, ++g) {
                    const int st = g % kPgStages;
                    const uint32_t ph = (g / kPgStages) & 1u;
                    const int ab = g & 1;
                    ok = mbar_wait(smem_u32(&bars->acc_empty[ab]), ((g >> 1) & 1u) ^ 1u, abort_flag, tmo, G.status);
                    if (ok) ok = mbar_wait(smem_u32(&bars->split[st]), ph, abort_flag, tmo, G.status);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t ah = smem_u32(base + st * kPgStageBytes);
                    const uint32_t al = ah + kPgHalf, phd = ah + 2 * kPgHalf, pl = ah + 3 * kPgHalf;
                    const uint32_t d_head = tmem + ab * 256, d_tail = d_head + 128;
#pragma unroll
                    for (int s = 0; s < 4; ++s) {
                        uint64_t dah, dal;
                        if (!G.trans) {
                            dah = make_sdesc_sw128(ah + s * 32, 16, 1024);
                            dal = make_sdesc_sw128(al + s * 32, 16, 1024);
                        } else {
                            dah = make_sdesc_mn32(ah + s * 1024);
                            dal = make_sdesc_mn32(al + s * 1024);
                        }
                        const uint64_t dph = make_sdesc_sw128(phd + s * 32, 16, 1024);
                        const uint64_t dpl = make_sdesc_sw128(pl + s * 32, 16, 1024);
                        mma_ss_tf32(d_tail, dal, dph, idesc, s > 0 ? 1u : 0u);
                        mma_ss_tf32(d_tail, dah, dpl, idesc, 1u);
                        mma_ss_tf32(d_head, dah, dph, idesc, s > 0 ? 1u : 0u);
                    }
                    tc_commit(smem_u32(&bars->empty[st]));
                    tc_commit(smem_u32(&bars->acc_full[ab]));
                }
            }
            if (g > 0) {
                // bounded wait for the last products before the CTA frees TMEM
                const int c = g - 1;
                const uint64_t t0 = globaltimer_ns();
                uint32_t spins = 0;
                while (!mbar_try_wait(smem_u32(&bars->acc_full[c & 1]), (c >> 1) & 1u)) {
                    if ((++spins & 63u) == 0u && globaltimer_ns() - t0 > tmo) {
                        record_error(G.status, ADA_ERR_TIMEOUT);
                        break;
                    }
                }
            }
        }
        __syncwarp();
    } else if (warp >= 4) {
        const int t = threadIdx.x - 128;
        const uint32_t lane_bits = static_cast<uint32_t>((warp & 3) * 32) << 16;
        const int rrow = (warp & 3) * 32 + lane;
        float acc[KP];
#pragma unroll
        for (int i = 0; i < KP; ++i) acc[i] = 0.f;
        auto add_chunk = [&](int g) -> bool {
            const int ab = g & 1;
            if (!mbar_wait(smem_u32(&bars->acc_full[ab]), (g >> 1) & 1u, abort_flag, tmo, G.status)) return false;
            tc_fence_after();
#pragma unroll
            for (int cc = 0; cc < KP / 16; ++cc) {
                uint32_t h[16], l[16];
                tmem_ld16(tmem + lane_bits + ab * 256 + cc * 16, h);
                tmem_ld16(tmem + lane_bits + ab * 256 + 128 + cc * 16, l);
                tmem_ld_wait();
                reg_fence16(h);
                reg_fence16(l);
#pragma unroll
                for (int i = 0; i < 16; ++i)
                    acc[cc * 16 + i] += __uint_as_float(h[i]) + __uint_as_float(l[i]);
            }
            tc_fence_before();
            mbar_arrive(smem_u32(&bars->acc_empty[ab]));
            return true;
        };
        auto store = [&](const PgItem& w) {
            const int grow = w.row0 + rrow;
            if (grow < G.rows) {
                float* o = G.out + w.b * G.out_bs + grow;
                if (G.splits == 1) {
#pragma unroll
                    for (int i = 0; i < KP; ++i)
                        if (i < G.k) o[i * G.ld_out] = acc[i];
                } else {
#pragma unroll
                    for (int i = 0; i < KP; ++i)
                        if (i < G.k) atomicAdd(o + i * G.ld_out, acc[i]);
                }
            }
#pragma unroll
            for (int i = 0; i < KP; ++i) acc[i] = 0.f;
        };
        int g = 0;
        bool ok = true, have_prev = false, prev_last = false;
        PgItem prev_item{};
        for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x) {
            const PgItem w = pg_item(G, it);
            for (int c = w.c0; c < w.c1; ++c, ++g) {
                const int st = g % kPgStages;
                ok = mbar_wait(smem_u32(&bars->full[st]), (g / kPgStages) & 1u, abort_flag, tmo, G.status);
                if (!ok) break;
                pg_split_stage<KP>(base + st * kPgStageBytes, t);
                mbar_arrive(smem_u32(&bars->split[st]));
                if (have_prev) {
                    ok = add_chunk(g - 1);
                    if (!ok) break;
                    if (prev_last) store(prev_item);
                }
                have_prev = true;
                prev_last = c == w.c1 - 1;
                prev_item = w;
            }
        }
        if (ok && have_prev) {
            ok = add_chunk(g - 1);
            if (ok && prev_last) store(prev_item);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// ---------------------------------------------------------------------------
// fp64 Gram of a panel: G[b] (upper triangle, zeroed by the caller) +=
// P[b][:, i0:i0+256] P[b][:, i0:i0+256]^T, 4x4 blocks per thread.
// ---------------------------------------------------------------------------
constexpr int kGramCols = 128;   // columns staged per pass (as fp64)
constexpr int kGramPasses = 4;   // passes per CTA before its atomics

__global__ void __launch_bounds__(256) gram64_kernel(const float* P, int64_t p_bs, int64_t p_ld, int k, int L,
                                                     double* G) {
    extern __shared__ double sgd[];  // [k][kGramCols + 1]
    constexpr int LD = kGramCols + 1;
    const int b = blockIdx.y;
    const float* src = P + b * p_bs;
    const int kb = (k + 3) / 4;
    const int npairs = kb * (kb + 1) / 2;
    // 4x4 blocks of the upper triangle: k <= 112 gives at most 406, two slots per thread
    constexpr int kSlots = 2;
    int bi_s[kSlots], bj_s[kSlots];
    double acc[kSlots][4][4];
#pragma unroll
    for (int sl = 0; sl < kSlots; ++sl) {
        const int pi = threadIdx.x + sl * blockDim.x;
        int bi = 0, rem = pi < npairs ? pi : 0;
        while (rem >= kb - bi) {
            rem -= kb - bi;
            ++bi;
        }
        bi_s[sl] = pi < npairs ? bi : -1;
        bj_s[sl] = bi + rem;
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int v = 0; v < 4; ++v) acc[sl][u][v] = 0.0;
    }
    for (int pass = 0; pass < kGramPasses; ++pass) {
        const int i0 = (blockIdx.x * kGramPasses + pass) * kGramCols;
        if (i0 >= L) break;
        const int w = min(kGramCols, L - i0);
        __syncthreads();
        for (int idx = threadIdx.x; idx < k * kGramCols; idx += blockDim.x) {
            const int c = idx / kGramCols, i = idx - c * kGramCols;
            sgd[c * LD + i] = i < w ? static_cast<double>(src[c * p_ld + i0 + i]) : 0.0;
        }
        __syncthreads();
#pragma unroll
        for (int sl = 0; sl < kSlots; ++sl) {
            if (bi_s[sl] < 0) continue;
            int ri[4], rj[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                ri[u] = min(4 * bi_s[sl] + u, k - 1) * LD;
                rj[u] = min(4 * bj_s[sl] + u, k - 1) * LD;
            }
            for (int i = 0; i < w; ++i) {
                double x[4], y[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    x[u] = sgd[ri[u] + i];
                    y[u] = sgd[rj[u] + i];
                }
#pragma unroll
                for (int u = 0; u < 4; ++u)
#pragma unroll
                    for (int v = 0; v < 4; ++v) acc[sl][u][v] = fma(x[u], y[v], acc[sl][u][v]);
            }
        }
    }
    double* g = G + static_cast<int64_t>(b) * k * k;
#pragma unroll
    for (int sl = 0; sl < kSlots; ++sl) {
        if (bi_s[sl] < 0) continue;
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int v = 0; v < 4; ++v) {
                const int r = 4 * bi_s[sl] + u, c = 4 * bj_s[sl] + v;
                if (r < k && c < k && r <= c) atomicAdd(g + r * k + c, acc[sl][u][v]);
            }
    }
}

// ---------------------------------------------------------------------------
// Cholesky G = R^T R (upper R, fp64) and X = R^-1, one CTA per matrix.
// A pivot at or below tau * G_jj marks column j as inside the span of the
// earlier ones: its row of R becomes e_j and its column of X is zero.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) chol_inv_kernel(const double* Gall, int k, double tau, double* Xall) {
    extern __shared__ double smd[];
    double* a = smd;          // [k][k], upper triangle
    double* x = smd + k * k;  // [k][k]
    __shared__ double gd[kMaxSketch];
    __shared__ int defic[kMaxSketch];
    const int b = blockIdx.x;
    const double* Gm = Gall + static_cast<int64_t>(b) * k * k;
    for (int idx = threadIdx.x; idx < k * k; idx += blockDim.x) {
        const int i = idx / k, j = idx - i * k;
        a[idx] = i <= j ? Gm[idx] : 0.0;
        x[idx] = 0.0;
    }
    for (int i = threadIdx.x; i < k; i += blockDim.x) gd[i] = Gm[i * k + i];
    __syncthreads();
    for (int j = 0; j < k; ++j) {
        if (threadIdx.x == 0) {
            const double d = a[j * k + j];
            const bool def = !(gd[j] > 0.0) || !(d > tau * gd[j]);
            defic[j] = def ? 1 : 0;
            a[j * k + j] = def ? 1.0 : sqrt(d);
        }
        __syncthreads();
        const double rjj = a[j * k + j];
        const bool def = defic[j] != 0;
        for (int l = j + 1 + threadIdx.x; l < k; l += blockDim.x) a[j * k + l] = def ? 0.0 : a[j * k + l] / rjj;
        __syncthreads();
        if (!def) {
            const int n = k - j - 1;
            for (int idx = threadIdx.x; idx < n * n; idx += blockDim.x) {
                const int p = j + 1 + idx / n, l = j + 1 + idx % n;
                if (l >= p) a[p * k + l] -= a[j * k + p] * a[j * k + l];
            }
        }
        __syncthreads();
    }
    for (int l = threadIdx.x; l < k; l += blockDim.x) {
        if (defic[l]) continue;
        x[l * k + l] = 1.0 / a[l * k + l];
        for (int p = l - 1; p >= 0; --p) {
            double s = 0.0;
            for (int t = p + 1; t <= l; ++t) s = fma(a[p * k + t], x[t * k + l], s);
            x[p * k + l] = -s / a[p * k + p];
        }
    }
    __syncthreads();
    double* X = Xall + static_cast<int64_t>(b) * k * k;
    for (int idx = threadIdx.x; idx < k * k; idx += blockDim.x) X[idx] = x[idx];
}

// ---------------------------------------------------------------------------
// Symmetric eigen-solve of W = B B^T (fp64 cyclic Jacobi, round-robin pairs),
// eigenvalues sorted descending: S = sqrt(lambda), MU = eigenvectors[:, :r],
// MV = MU / S (zero where S is zero). One CTA per matrix.
// ---------------------------------------------------------------------------
constexpr int kEigThreads = 1024;
constexpr size_t kSvdSmemMax = 200 * 1024;

__device__ double block_sum(double v, double* red) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    double s = 0.0;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) s += red[w];
    return s;
}

// Round-robin pairing: in round `round`, slot x meets slot kk-1-x; slot kk-1
// stays put and the others rotate.
__device__ __forceinline__ void rr_pair(int kk, int round, int pi, int* p, int* q) {
    const int x0 = pi, x1 = kk - 1 - pi;
    int a = x0 == kk - 1 ? kk - 1 : (x0 + round) % (kk - 1);
    int b = x1 == kk - 1 ? kk - 1 : (x1 + round) % (kk - 1);
    *p = a < b ? a : b;
    *q = a < b ? b : a;
}

// 1/sqrt(x) and 1/x for x within the float range: an fp32 estimate refined
// by two Newton steps in fp64 (y <- y (3 - x y^2) / 2, y <- y (2 - x y)),
// each of which squares the relative error.
__device__ __forceinline__ double rsqrt_newton(double x) {
    double y = static_cast<double>(rsqrtf(static_cast<float>(x)));
    y = y * fma(-0.5 * x * y, y, 1.5);
    y = y * fma(-0.5 * x * y, y, 1.5);
    return y;
}
__device__ __forceinline__ double rcp_newton(double x) {
    double y = static_cast<double>(__frcp_rn(static_cast<float>(x)));
    y = y * fma(-x, y, 2.0);
    y = y * fma(-x, y, 2.0);
    return y;
}

// Jacobi rotation (c, s) that zeroes a_pq: t = sign(d) e / (|d| + sqrt(d^2 +
// e^2)) with d = a_qq - a_pp, e = 2 a_pq (the smaller root of
// t^2 + 2 (d/e) t - 1 = 0), c = 1/sqrt(1 + t^2), s = t c. d and e are first
// scaled by a power of two so every intermediate sits well inside the
// float range of the Newton seeds.
__device__ __forceinline__ void jacobi_rotation(double app, double aqq, double apq, double* c, double* s) {
    const double d = aqq - app, e = 2.0 * apq;
    const int ex = ilogb(fmax(fabs(d), fabs(e)));
    const double ds = scalbn(d, -ex), es = scalbn(e, -ex);  // max(|ds|, |es|) in [1, 2)
    const double h = fma(ds, ds, es * es);                  // in [1, 8)
    const double r = h * rsqrt_newton(h);
    const double t = (d >= 0.0 ? es : -es) * rcp_newton(fabs(ds) + r);
    *c = rsqrt_newton(fma(t, t, 1.0));
    *s = t * *c;
}

// Round structure: the rotations of all disjoint pairs are formed in
// parallel (one thread each), then every (pair, column) element of the two
// rows is updated by its own thread, and after a block barrier every
// (pair, row) element of the two columns of W and V.
__global__ void __launch_bounds__(kEigThreads) eig_kernel(const double* Wall, int k, int r, float* s_out,
                                                          int64_t s_bs, int64_t s_st, double* mu_all,
                                                          double* mv_all, int max_sweeps) {
    extern __shared__ double smd[];
    const int kk = k + (k & 1);
    const int ld = kk + 1;
    double* a = smd;            // [kk][ld]
    double* v = smd + kk * ld;  // [kk][ld]
    __shared__ double cs_c[kMaxSketch / 2], cs_s[kMaxSketch / 2];
    __shared__ double red[kEigThreads / 32];
    __shared__ int2 pq[kMaxSketch / 2];
    const int b = blockIdx.x;
    const double* W = Wall + static_cast<int64_t>(b) * k * k;
    for (int idx = threadIdx.x; idx < kk * kk; idx += blockDim.x) {
        const int i = idx / kk, j = idx - i * kk;
        double val = 0.0;
        if (i < k && j < k) val = i <= j ? W[i * k + j] : W[j * k + i];
        a[i * ld + j] = val;
        v[i * ld + j] = i == j ? 1.0 : 0.0;
    }
    __syncthreads();
    const int half = kk / 2;
    for (int sweep = 0; sweep < max_sweeps; ++sweep) {
        double off = 0.0, dg = 0.0;
        for (int idx = threadIdx.x; idx < kk * kk; idx += blockDim.x) {
            const int i = idx / kk, j = idx - i * kk;
            const double e = a[i * ld + j] * a[i * ld + j];
            if (i == j) dg += e; else off += e;
        }
        off = block_sum(off, red);
        dg = block_sum(dg, red);
        if (!(off > 1e-28 * dg)) break;
        // Rotations are skipped once |a_pq| is within 100x of the rounding
        // level next to its diagonal pair or next to the matrix norm (below
        // that a rotation only moves rounding noise around); a sweep without
        // any rotation ends the iteration.
        const double tiny = 1e-14 * sqrt(dg);
        int rotated = 0;
        for (int round = 0; round < kk - 1; ++round) {
            for (int pi = threadIdx.x; pi < half; pi += blockDim.x) {
                int p, q;
                rr_pair(kk, round, pi, &p, &q);
                double c = 1.0, s = 0.0;
                const double apq = a[p * ld + q], app = a[p * ld + p], aqq = a[q * ld + q];
                // |a_pq| > 1e-14 sqrt(|a_pp a_qq|), compared squared
                if (fabs(apq) > tiny && apq * apq > 1e-28 * fabs(app * aqq)) {
                    jacobi_rotation(app, aqq, apq, &c, &s);
                    rotated |= s != 0.0;
                }
                cs_c[pi] = c;
                cs_s[pi] = s;
                pq[pi] = make_int2(p, q);
            }
            __syncthreads();
            for (int idx = threadIdx.x; idx < half * kk; idx += blockDim.x) {
                const int pi = idx / kk, x = idx - pi * kk;
                const double s = cs_s[pi];
                if (s != 0.0) {
                    const double c = cs_c[pi];
                    const int p = pq[pi].x, q = pq[pi].y;
                    const double ap = a[p * ld + x], aq = a[q * ld + x];
                    a[p * ld + x] = c * ap - s * aq;
                    a[q * ld + x] = s * ap + c * aq;
                }
            }
            __syncthreads();
            for (int idx = threadIdx.x; idx < half * kk; idx += blockDim.x) {
                const int pi = idx / kk, x = idx - pi * kk;
                const double s = cs_s[pi];
                if (s == 0.0) continue;
                const double c = cs_c[pi];
                const int p = pq[pi].x, q = pq[pi].y;
                const double ap = a[x * ld + p], aq = a[x * ld + q];
                a[x * ld + p] = c * ap - s * aq;
                a[x * ld + q] = s * ap + c * aq;
                const double vp = v[x * ld + p], vq = v[x * ld + q];
                v[x * ld + p] = c * vp - s * vq;
                v[x * ld + q] = s * vp + c * vq;
            }
            __syncthreads();
        }
        if (!__syncthreads_or(rotated)) break;
    }
    for (int i = threadIdx.x; i < k; i += blockDim.x) {
        const double d = a[i * ld + i];
        int rank = 0;
        double dmax = 0.0;
        for (int j = 0; j < k; ++j) {
            const double e = a[j * ld + j];
            if (e > d || (e == d && j < i)) ++rank;
            dmax = fmax(dmax, e);
        }
        if (rank >= r) continue;
        const double sv = d > 0.0 ? sqrt(d) : 0.0;
        s_out[b * s_bs + rank * s_st] = static_cast<float>(sv);
        // Directions 1e-12 below the largest singular value are rounding
        // noise of the fp32 inputs; their Vh rows are left zero.
        const double inv = sv > 1e-12 * sqrt(dmax) ? 1.0 / sv : 0.0;
        double* mu = mu_all + static_cast<int64_t>(b) * k * r;
        double* mv = mv_all + static_cast<int64_t>(b) * k * r;
        for (int c = 0; c < k; ++c) {
            mu[c * r + rank] = v[c * ld + i];
            mv[c * r + rank] = v[c * ld + i] * inv;
        }
    }
}

// ---------------------------------------------------------------------------
// One-sided (Hestenes) Jacobi SVD of B = Q^T A, k x n, in fp64: pairs of rows
// are rotated until all rows are mutually orthogonal, so B = R diag(S) Z^T
// with R the accumulated k x k rotation and the rows of Z unit vectors. One
// half-warp per pair of each round-robin round (dot products, rotation, both
// rows, both columns of R), one block barrier per round. Working on B
// itself, not on B B^T, keeps the small singular values' relative accuracy.
// Writes S (the r largest, descending), mu = R[:, those] (k x r; U = Q mu)
// and Vh's rows (Z's rows; zero where S <= 1e-12 S_max, as for the Gram path).
// ---------------------------------------------------------------------------
constexpr int kSvdThreads = 1024;  // 64 half-warps >= kMaxSketch / 2 pairs

size_t svdj_smem(int k, int64_t n) {
    const int kk = k + (k & 1);
    return (static_cast<size_t>(kk) * (n + 1) + static_cast<size_t>(kk) * (kk + 1)) * sizeof(double);
}

__global__ void __launch_bounds__(kSvdThreads) svdj_kernel(const float* zall, int64_t z_bs, int64_t z_ld, int k,
                                                           int n, int r, float* s_out, int64_t s_bs, int64_t s_st,
                                                           double* mu_all, float* vh, int64_t vh_bs, int64_t vh_rs,
                                                           int64_t vh_cs, int max_sweeps) {
    extern __shared__ double smd[];
    const int kk = k + (k & 1);
    const int ldb = n + 1, ldr = kk + 1;
    double* bm = smd;              // [kk][ldb] rows of B, rotated in place
    double* rm = smd + kk * ldb;   // [kk][ldr] R
    __shared__ double sig[kMaxSketch + 1];
    __shared__ int by_rank[kMaxSketch + 1];
    const int b = blockIdx.x;
    const float* z = zall + static_cast<int64_t>(b) * z_bs;
    for (int idx = threadIdx.x; idx < kk * n; idx += kSvdThreads) {
        const int i = idx / n, j = idx - i * n;
        bm[i * ldb + j] = i < k ? static_cast<double>(z[i * z_ld + j]) : 0.0;
    }
    for (int idx = threadIdx.x; idx < kk * kk; idx += kSvdThreads) {
        const int i = idx / kk, j = idx - i * kk;
        rm[i * ldr + j] = i == j ? 1.0 : 0.0;
    }
    __syncthreads();
    const int half = kk / 2;
    const int hw = threadIdx.x >> 4, hl = threadIdx.x & 15;
    const unsigned hmask = (threadIdx.x & 16) ? 0xffff0000u : 0x0000ffffu;
    for (int sweep = 0; sweep < max_sweeps; ++sweep) {
        int rotated = 0;
        for (int round = 0; round < kk - 1; ++round) {
            if (hw < half) {
                int p, q;
                rr_pair(kk, round, hw, &p, &q);
                double al = 0.0, be = 0.0, ga = 0.0;
                for (int j = hl; j < n; j += 16) {
                    const double x = bm[p * ldb + j], y = bm[q * ldb + j];
                    al = fma(x, x, al);
                    be = fma(y, y, be);
                    ga = fma(x, y, ga);
                }
#pragma unroll
                for (int o = 8; o > 0; o >>= 1) {
                    al += __shfl_xor_sync(hmask, al, o);
                    be += __shfl_xor_sync(hmask, be, o);
                    ga += __shfl_xor_sync(hmask, ga, o);
                }
                // rotate unless |b_p . b_q| <= 1e-15 |b_p| |b_q|
                if (ga != 0.0 && ga * ga > 1e-30 * al * be) {
                    double c, s;
                    jacobi_rotation(al, be, ga, &c, &s);
                    if (s != 0.0) {
                        rotated = 1;
                        for (int j = hl; j < n; j += 16) {
                            const double x = bm[p * ldb + j], y = bm[q * ldb + j];
                            bm[p * ldb + j] = c * x - s * y;
                            bm[q * ldb + j] = s * x + c * y;
                        }
                        for (int i = hl; i < kk; i += 16) {
                            const double x = rm[i * ldr + p], y = rm[i * ldr + q];
                            rm[i * ldr + p] = c * x - s * y;
                            rm[i * ldr + q] = s * x + c * y;
                        }
                    }
                }
            }
            __syncthreads();
        }
        if (!__syncthreads_or(rotated)) break;
    }
    // singular values: the row norms
    for (int i = hw; i < k; i += kSvdThreads / 16) {
        double a2 = 0.0;
        for (int j = hl; j < n; j += 16) a2 = fma(bm[i * ldb + j], bm[i * ldb + j], a2);
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) a2 += __shfl_xor_sync(hmask, a2, o);
        if (hl == 0) sig[i] = sqrt(a2);
    }
    __syncthreads();
    if (threadIdx.x < k) {
        const int i = threadIdx.x;
        const double d = sig[i];
        int rank = 0;
        for (int j = 0; j < k; ++j) {
            const double e = sig[j];
            if (e > d || (e == d && j < i)) ++rank;
        }
        if (rank < r) {
            by_rank[rank] = i;
            s_out[b * s_bs + rank * s_st] = static_cast<float>(d);
            double* mu = mu_all + static_cast<int64_t>(b) * k * r;
            for (int c = 0; c < k; ++c) mu[c * r + rank] = rm[c * ldr + i];
        }
    }
    __syncthreads();
    double smax = 0.0;
    for (int j = 0; j < k; ++j) smax = fmax(smax, sig[j]);
    for (int idx = threadIdx.x; idx < r * n; idx += kSvdThreads) {
        const int rank = idx / n, j = idx - rank * n;
        const int i = by_rank[rank];
        const double sv = sig[i];
        const double val = sv > 1e-12 * smax ? bm[i * ldb + j] / sv : 0.0;
        vh[b * vh_bs + rank * vh_rs + j * vh_cs] = static_cast<float>(val);
    }
}

// ---------------------------------------------------------------------------
// out(i, c) = sum_{c'} P[c'][i] * M[c'][c] for c < nc (c' <= c when
// triangular), one output row i per thread; fp64 or fp32 accumulation.
// ---------------------------------------------------------------------------
struct ApplyArgs {
    const float* P;
    int64_t p_bs, p_ld;
    int k, L;
    const double* M;
    int64_t m_bs;
    int nc, tri;
    float* out;
    int64_t o_bs, o_sc, o_si;
};

template <typename Acc>
__global__ void __launch_bounds__(128) panel_apply_kernel(const __grid_constant__ ApplyArgs A) {
    extern __shared__ double smd[];
    const int ncp = (A.nc + 15) & ~15;
    Acc* sM = reinterpret_cast<Acc*>(smd);                  // [k][ncp], zero padded
    float* sP = reinterpret_cast<float*>(sM + A.k * ncp);  // [k][128]
    const int b = blockIdx.y;
    const int i0 = blockIdx.x * 128;
    const int i = i0 + threadIdx.x;
    const double* M = A.M + b * A.m_bs;
    for (int idx = threadIdx.x; idx < A.k * ncp; idx += blockDim.x) {
        const int cp = idx / ncp, c = idx - cp * ncp;
        sM[idx] = c < A.nc ? static_cast<Acc>(M[cp * A.nc + c]) : Acc(0);
    }
    const float* P = A.P + b * A.p_bs;
    for (int c = 0; c < A.k; ++c) sP[c * 128 + threadIdx.x] = i < A.L ? P[c * A.p_ld + i] : 0.f;
    __syncthreads();
    if (i >= A.L) return;
    float* o = A.out + b * A.o_bs + i * A.o_si;
    for (int c0 = 0; c0 < A.nc; c0 += 16) {
        Acc acc[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[j] = Acc(0);
        const int lim = A.tri ? min(c0 + 16, A.k) : A.k;
        for (int cp = 0; cp < lim; ++cp) {
            const Acc pv = static_cast<Acc>(sP[cp * 128 + threadIdx.x]);
            const Acc* mrow = sM + cp * ncp + c0;
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[j] = fma(pv, mrow[j], acc[j]);
        }
#pragma unroll
        for (int j = 0; j < 16; ++j)
            if (c0 + j < A.nc) o[(c0 + j) * A.o_sc] = static_cast<float>(acc[j]);
    }
}

// dst[b][c][i] = src(b, i, c) (a [batch, rows, cols] view into a [cols, ld] panel)
__global__ void to_panel_kernel(const float* src, int64_t sb, int64_t s0, int64_t s1, int64_t batch, int rows,
                                int cols, float* dst, int64_t d_bs, int64_t d_ld) {
    const int64_t total = batch * rows * cols;
    for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
         t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t b = t / (static_cast<int64_t>(rows) * cols);
        const int64_t rem = t - b * rows * cols;
        const int c = static_cast<int>(rem / rows), i = static_cast<int>(rem % rows);
        dst[b * d_bs + c * d_ld + i] = src[b * sb + i * s0 + c * s1];
    }
}

// dst[b][i][j] (row stride ld) = src(b, i, j)
__global__ void copy_rows_kernel(const float* src, int64_t sb, int64_t s0, int64_t s1, int64_t batch, int rows,
                                 int cols, float* dst, int64_t ld) {
    const int64_t total = batch * rows * cols;
    for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
         t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t b = t / (static_cast<int64_t>(rows) * cols);
        const int64_t rem = t - b * rows * cols;
        const int i = static_cast<int>(rem / cols), j = static_cast<int>(rem % cols);
        dst[(b * rows + i) * ld + j] = src[b * sb + i * s0 + j * s1];
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
int fail_msg(int code, const char* fmt, long long a = 0, long long b = 0) {
    char buf[256];
    snprintf(buf, sizeof(buf), fmt, a, b);
    return record_last_error(code, buf);
}

int64_t round4(int64_t x) { return (x + 3) & ~int64_t(3); }
size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct RsvdPlan {
    int64_t batch, m, n, m4, n4;
    int k, r, kp;
    bool copy_a;
    size_t off_a, off_om, off_y, off_z, off_q, off_g, off_x, off_mu, off_mv, total;
};

bool a_tma_ok(const AdaTensor* a) {
    if ((reinterpret_cast<uintptr_t>(a->data) & 15u) != 0) return false;
    if (a->stride[2] != 1 && a->shape[2] > 1) return false;
    if (a->shape[1] > 1 && (a->stride[1] <= 0 || (a->stride[1] * 4) % 16 != 0)) return false;
    if (a->shape[0] > 1 && (a->stride[0] <= 0 || (a->stride[0] * 4) % 16 != 0)) return false;
    return true;
}

int rsvd_plan(const AdaTensor* a, const AdaTensor* omega, int rank, RsvdPlan* P) {
    if (a == nullptr || omega == nullptr || a->data == nullptr || omega->data == nullptr)
        return fail_msg(ADA_ERR_INVALID, "a and omega are required");
    if (a->dtype != ADA_F32 || omega->dtype != ADA_F32)
        return fail_msg(ADA_ERR_DTYPE, "randomized SVD takes fp32 a and omega");
    if (a->ndim != 3 || omega->ndim != 3) return fail_msg(ADA_ERR_SHAPE, "a is [batch, m, n], omega [batch, n, k]");
    std::memset(P, 0, sizeof(*P));
    P->batch = a->shape[0];
    P->m = a->shape[1];
    P->n = a->shape[2];
    if (P->batch < 1 || P->m < 1 || P->n < 1) return fail_msg(ADA_ERR_SHAPE, "empty matrix");
    if (P->batch > 65535 || P->m > (1 << 30) || P->n > (1 << 30))
        return fail_msg(ADA_ERR_UNSUPPORTED, "batch %lld or matrix extents too large", P->batch);
    if (omega->shape[0] != P->batch || omega->shape[1] != P->n)
        return fail_msg(ADA_ERR_SHAPE, "omega must be [batch, n, k]");
    const int64_t k = omega->shape[2];
    const int64_t mn = P->m < P->n ? P->m : P->n;
    if (rank < 1 || rank > k) return fail_msg(ADA_ERR_INVALID, "rank %lld outside [1, k=%lld]", rank, k);
    if (k > mn) return fail_msg(ADA_ERR_SHAPE, "sketch width %lld exceeds min(m, n) = %lld", k, mn);
    if (k > kMaxSketch) return fail_msg(ADA_ERR_UNSUPPORTED, "sketch width %lld above %lld", k, kMaxSketch);
    P->k = static_cast<int>(k);
    P->r = rank;
    P->kp = k <= 32 ? 32 : static_cast<int>((k + 15) / 16 * 16);  // MMA N, a multiple of 16
    P->m4 = round4(P->m);
    P->n4 = round4(P->n);
    P->copy_a = !a_tma_ok(a);
    const size_t B = static_cast<size_t>(P->batch);
    size_t off = 0;
    P->off_a = off;
    if (P->copy_a) off = align256(off + B * P->m * P->n4 * 4);
    P->off_om = off;
    off = align256(off + B * k * P->n4 * 4);
    P->off_y = off;
    off = align256(off + B * k * P->m4 * 4);
    P->off_z = off;
    off = align256(off + B * k * P->n4 * 4);
    P->off_q = off;
    off = align256(off + B * k * P->m4 * 4);
    P->off_g = off;
    off = align256(off + B * k * k * 8);
    P->off_x = off;
    off = align256(off + B * k * k * 8);
    P->off_mu = off;
    off = align256(off + B * k * rank * 8);
    P->off_mv = off;
    off = align256(off + B * k * rank * 8);
    P->total = off;
    return ADA_OK;
}

int encode3d(CUtensorMap* map, const void* base, int64_t d0, int64_t d1, int64_t d2, int64_t s1_bytes,
             int64_t s2_bytes, uint32_t box0, uint32_t box1,
             CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
    PFN_cuTensorMapEncodeTiled_v12000 enc;
    int rc = tensor_map_encoder(&enc);
    if (rc) return rc;
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(d0), static_cast<cuuint64_t>(d1), static_cast<cuuint64_t>(d2)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(s1_bytes > 0 ? s1_bytes : 16),
                             static_cast<cuuint64_t>(s2_bytes > 0 ? s2_bytes : 16)};
    cuuint32_t box[3] = {box0, box1, 1};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail_msg(ADA_ERR_LAYOUT, "cuTensorMapEncodeTiled failed (%lld)", static_cast<int>(r));
    return ADA_OK;
}

constexpr int kPgSmem = kPgStages * kPgStageBytes + 1024 + 256;

struct RsvdCtx {
    const RsvdPlan* P;
    const float* a;   // A base used by the GEMMs
    int64_t a_bs, a_ld;
    uint8_t* ws;
    unsigned int* status;
    cudaStream_t s;
};

// out panel (ld out_ld, rows `rows`) = (A X)^T or (A^T Y)^T with input panel
// `in` of width in_L (row stride in_ld).
int run_panel_gemm(const RsvdCtx& C, int trans, const float* in, int64_t in_L, int64_t in_ld, float* out,
                   int64_t out_ld) {
    const RsvdPlan& P = *C.P;
    PanelGemm G;
    std::memset(&G, 0, sizeof(G));
    int rc;
    if ((rc = encode3d(&G.ta, C.a, P.n, P.m, P.batch, C.a_ld * 4, C.a_bs * 4, 32, trans ? 32 : 128,
                       trans ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B)))
        return rc;
    if ((rc = encode3d(&G.tp, in, in_L, P.k, P.batch, in_ld * 4, static_cast<int64_t>(P.k) * in_ld * 4, 32,
                       static_cast<uint32_t>(P.kp))))
        return rc;
    G.out = out;
    G.out_bs = static_cast<int64_t>(P.k) * out_ld;
    G.ld_out = out_ld;
    G.rows = static_cast<int>(trans ? P.n : P.m);
    G.kdim = static_cast<int>(trans ? P.m : P.n);
    G.k = P.k;
    G.kp = P.kp;
    G.trans = trans;
    G.status = C.status;
    G.timeout_ns = default_wait_timeout_ns();
    // Work items: enough (batch, tile, K split) items to give every SM two;
    // the K dimension is split only when the tiles alone are too few.
    int sms = 0, dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
        return fail_msg(ADA_ERR_CUDA, "device query failed");
    G.batch = static_cast<int>(P.batch);
    G.tiles = (G.rows + 127) / 128;
    const int nchunks = (G.kdim + 31) / 32;
    const int64_t tiles_total = static_cast<int64_t>(G.batch) * G.tiles;
    int splits = 1;
    if (tiles_total < 2 * sms) splits = static_cast<int>((2 * sms + tiles_total - 1) / tiles_total);
    if (splits > nchunks) splits = nchunks;
    G.cps = (nchunks + splits - 1) / splits;
    G.splits = (nchunks + G.cps - 1) / G.cps;
    if (G.splits > 1 &&
        cudaMemsetAsync(out, 0, static_cast<size_t>(P.batch) * P.k * out_ld * sizeof(float), C.s) != cudaSuccess)
        return fail_msg(ADA_ERR_CUDA, "clearing a panel failed");
    const int64_t items = tiles_total * G.splits;
    if (items > (int64_t(1) << 31) - 1) return fail_msg(ADA_ERR_UNSUPPORTED, "too many work items");
    const dim3 grid(static_cast<unsigned>(items < sms ? items : sms));
    switch (P.kp) {
        case 32: panel_gemm_kernel<32><<<grid, kPgThreads, kPgSmem, C.s>>>(G); break;
        case 48: panel_gemm_kernel<48><<<grid, kPgThreads, kPgSmem, C.s>>>(G); break;
        case 64: panel_gemm_kernel<64><<<grid, kPgThreads, kPgSmem, C.s>>>(G); break;
        case 80: panel_gemm_kernel<80><<<grid, kPgThreads, kPgSmem, C.s>>>(G); break;
        case 96: panel_gemm_kernel<96><<<grid, kPgThreads, kPgSmem, C.s>>>(G); break;
        case 112: panel_gemm_kernel<112><<<grid, kPgThreads, kPgSmem, C.s>>>(G); break;
        default: return fail_msg(ADA_ERR_UNSUPPORTED, "panel width %lld", P.kp);
    }
    return cudaGetLastError() == cudaSuccess ? ADA_OK : fail_msg(ADA_ERR_LAUNCH, "panel GEMM launch failed");
}

int run_gram(const RsvdCtx& C, const float* panel, int64_t L, int64_t ld, double* g) {
    const RsvdPlan& P = *C.P;
    const size_t bytes = static_cast<size_t>(P.batch) * P.k * P.k * 8;
    if (cudaMemsetAsync(g, 0, bytes, C.s) != cudaSuccess) return fail_msg(ADA_ERR_CUDA, "clearing a Gram failed");
    const size_t smem = static_cast<size_t>(P.k) * (kGramCols + 1) * 8;
    const int64_t per_cta = static_cast<int64_t>(kGramCols) * kGramPasses;
    const dim3 grid(static_cast<unsigned>((L + per_cta - 1) / per_cta), static_cast<unsigned>(P.batch));
    gram64_kernel<<<grid, 256, smem, C.s>>>(panel, static_cast<int64_t>(P.k) * ld, ld, P.k, static_cast<int>(L), g);
    return cudaGetLastError() == cudaSuccess ? ADA_OK : fail_msg(ADA_ERR_LAUNCH, "Gram launch failed");
}

int run_chol(const RsvdCtx& C, const double* g, double* x) {
    const RsvdPlan& P = *C.P;
    const size_t smem = static_cast<size_t>(2) * P.k * P.k * 8;
    chol_inv_kernel<<<static_cast<unsigned>(P.batch), 256, smem, C.s>>>(g, P.k, 1e-14, x);
    return cudaGetLastError() == cudaSuccess ? ADA_OK : fail_msg(ADA_ERR_LAUNCH, "Cholesky launch failed");
}

template <typename Acc>
int run_apply(const RsvdCtx& C, const float* panel, int64_t L, int64_t ld, const double* M, int nc, int tri,
              float* out, int64_t o_bs, int64_t o_sc, int64_t o_si) {
    const RsvdPlan& P = *C.P;
    ApplyArgs A;
    A.P = panel;
    A.p_bs = static_cast<int64_t>(P.k) * ld;
    A.p_ld = ld;
    A.k = P.k;
    A.L = static_cast<int>(L);
    A.M = M;
    A.m_bs = static_cast<int64_t>(P.k) * nc;
    A.nc = nc;
    A.tri = tri;
    A.out = out;
    A.o_bs = o_bs;
    A.o_sc = o_sc;
    A.o_si = o_si;
    const size_t smem = static_cast<size_t>(P.k) * ((nc + 15) & ~15) * sizeof(Acc) + static_cast<size_t>(P.k) * 128 * 4;
    const dim3 grid(static_cast<unsigned>((L + 127) / 128), static_cast<unsigned>(P.batch));
    panel_apply_kernel<Acc><<<grid, 128, smem, C.s>>>(A);
    return cudaGetLastError() == cudaSuccess ? ADA_OK : fail_msg(ADA_ERR_LAUNCH, "panel apply launch failed");
}

template <typename K>
int allow_smem(K kern, size_t bytes) {
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)) ==
                   cudaSuccess
               ? ADA_OK
               : fail_msg(ADA_ERR_LAUNCH, "shared-memory opt-in failed");
}

}  // namespace
}  // namespace ada

using namespace ada;

extern "C" size_t ada_rsvd_workspace_bytes(const AdaTensor* a, const AdaTensor* omega, int32_t rank) {
    RsvdPlan P;
    if (rsvd_plan(a, omega, rank, &P) != ADA_OK) return 0;
    return P.total;
}

extern "C" int ada_rsvd(const AdaTensor* a, const AdaTensor* omega, int32_t rank, int32_t n_power, AdaTensor* u,
                        AdaTensor* s, AdaTensor* vh, void* workspace, size_t workspace_bytes, void* stream) {
    unsigned int* st;
    int rc = device_status_word(&st);
    if (rc) return rc;
    RsvdPlan P;
    if ((rc = rsvd_plan(a, omega, rank, &P))) return rc;
    if (n_power < 0 || n_power > 64) return fail_msg(ADA_ERR_INVALID, "power iterations %lld", n_power);
    if (u == nullptr || s == nullptr || vh == nullptr || u->data == nullptr || s->data == nullptr ||
        vh->data == nullptr)
        return fail_msg(ADA_ERR_INVALID, "u, s and vh are required");
    if (u->dtype != ADA_F32 || s->dtype != ADA_F32 || vh->dtype != ADA_F32)
        return fail_msg(ADA_ERR_DTYPE, "u, s, vh must be fp32");
    if (u->ndim != 3 || u->shape[0] != P.batch || u->shape[1] != P.m || u->shape[2] != rank)
        return fail_msg(ADA_ERR_SHAPE, "u must be [batch, m, rank]");
    if (s->ndim != 2 || s->shape[0] != P.batch || s->shape[1] != rank)
        return fail_msg(ADA_ERR_SHAPE, "s must be [batch, rank]");
    if (vh->ndim != 3 || vh->shape[0] != P.batch || vh->shape[1] != rank || vh->shape[2] != P.n)
        return fail_msg(ADA_ERR_SHAPE, "vh must be [batch, rank, n]");
    if (workspace == nullptr || workspace_bytes < P.total)
        return fail_msg(ADA_ERR_WORKSPACE, "workspace of %lld bytes needed, %lld given", static_cast<long long>(P.total),
                        static_cast<long long>(workspace_bytes));
    if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
        return fail_msg(ADA_ERR_LAYOUT, "workspace must be 256-byte aligned");
    if ((rc = allow_smem(panel_gemm_kernel<32>, kPgSmem)) || (rc = allow_smem(panel_gemm_kernel<48>, kPgSmem)) ||
        (rc = allow_smem(panel_gemm_kernel<64>, kPgSmem)) || (rc = allow_smem(panel_gemm_kernel<80>, kPgSmem)) ||
        (rc = allow_smem(panel_gemm_kernel<96>, kPgSmem)) || (rc = allow_smem(panel_gemm_kernel<112>, kPgSmem)) ||
        (rc = allow_smem(gram64_kernel, static_cast<size_t>(P.k) * (kGramCols + 1) * 8)) ||
        (rc = allow_smem(chol_inv_kernel, static_cast<size_t>(2) * P.k * P.k * 8)) ||
        (rc = allow_smem(eig_kernel, static_cast<size_t>(2) * (P.k + 1) * (P.k + 2) * 8)) ||
        (svdj_smem(P.k, P.n) <= kSvdSmemMax && (rc = allow_smem(svdj_kernel, svdj_smem(P.k, P.n)))) ||
        (rc = allow_smem(panel_apply_kernel<double>,
                         static_cast<size_t>(P.k) * ((P.k + 15) & ~15) * 8 + static_cast<size_t>(P.k) * 128 * 4)) ||
        (rc = allow_smem(panel_apply_kernel<float>,
                         static_cast<size_t>(P.k) * ((P.k + 15) & ~15) * 4 + static_cast<size_t>(P.k) * 128 * 4)))
        return rc;

    cudaStream_t strm = static_cast<cudaStream_t>(stream);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    RsvdCtx C;
    C.P = &P;
    C.ws = ws;
    C.status = st;
    C.s = strm;
    const int64_t k = P.k;
    if (P.copy_a) {
        float* ac = reinterpret_cast<float*>(ws + P.off_a);
        copy_rows_kernel<<<1184, 256, 0, strm>>>(static_cast<const float*>(a->data), a->stride[0], a->stride[1],
                                                 a->stride[2], P.batch, static_cast<int>(P.m),
                                                 static_cast<int>(P.n), ac, P.n4);
        if (cudaGetLastError() != cudaSuccess) return fail_msg(ADA_ERR_LAUNCH, "copy launch failed");
        C.a = ac;
        C.a_ld = P.n4;
        C.a_bs = P.m * P.n4;
    } else {
        C.a = static_cast<const float*>(a->data);
        C.a_ld = P.m > 1 ? a->stride[1] : P.n4;
        C.a_bs = P.batch > 1 ? a->stride[0] : P.m * C.a_ld;
    }
    float* om = reinterpret_cast<float*>(ws + P.off_om);
    float* y = reinterpret_cast<float*>(ws + P.off_y);
    float* z = reinterpret_cast<float*>(ws + P.off_z);
    float* q = reinterpret_cast<float*>(ws + P.off_q);
    double* g = reinterpret_cast<double*>(ws + P.off_g);
    double* x = reinterpret_cast<double*>(ws + P.off_x);
    double* mu = reinterpret_cast<double*>(ws + P.off_mu);
    double* mv = reinterpret_cast<double*>(ws + P.off_mv);

    to_panel_kernel<<<592, 256, 0, strm>>>(static_cast<const float*>(omega->data), omega->stride[0],
                                           omega->stride[1], omega->stride[2], P.batch, static_cast<int>(P.n),
                                           P.k, om, k * P.n4, P.n4);
    if (cudaGetLastError() != cudaSuccess) return fail_msg(ADA_ERR_LAUNCH, "sketch transpose launch failed");
    // Y = A Omega; power iterations Y = A (A^T Y)  (low_rank.py:86-90)
    if ((rc = run_panel_gemm(C, 0, om, P.n, P.n4, y, P.m4))) return rc;
    for (int it = 0; it < n_power; ++it) {
        if ((rc = run_panel_gemm(C, 1, y, P.m, P.m4, z, P.n4))) return rc;
        if ((rc = run_panel_gemm(C, 0, z, P.n, P.n4, y, P.m4))) return rc;
    }
    // Q = orth(Y): CholeskyQR twice (pass 1 accumulates in fp64)
    if ((rc = run_gram(C, y, P.m, P.m4, g)) || (rc = run_chol(C, g, x)) ||
        (rc = run_apply<double>(C, y, P.m, P.m4, x, P.k, 1, q, k * P.m4, P.m4, 1)))
        return rc;
    if ((rc = run_gram(C, q, P.m, P.m4, g)) || (rc = run_chol(C, g, x)) ||
        (rc = run_apply<float>(C, q, P.m, P.m4, x, P.k, 1, y, k * P.m4, P.m4, 1)))
        return rc;
    // B = Q^T A  (low_rank.py:96): the panel of (A^T Q)^T is B itself
    if ((rc = run_panel_gemm(C, 1, y, P.m, P.m4, z, P.n4))) return rc;
    const size_t sv_smem = svdj_smem(P.k, P.n);
    if (sv_smem <= kSvdSmemMax) {
        // SVD of B by one-sided Jacobi; U = Q R[:, :r]  (low_rank.py:99-107)
        svdj_kernel<<<static_cast<unsigned>(P.batch), kSvdThreads, sv_smem, strm>>>(
            z, k * P.n4, P.n4, P.k, static_cast<int>(P.n), rank, static_cast<float*>(s->data), s->stride[0],
            s->stride[1], mu, static_cast<float*>(vh->data), vh->stride[0], vh->stride[1], vh->stride[2], 30);
        if (cudaGetLastError() != cudaSuccess) return fail_msg(ADA_ERR_LAUNCH, "Jacobi SVD launch failed");
        return run_apply<float>(C, y, P.m, P.m4, mu, rank, 0, static_cast<float*>(u->data), u->stride[0],
                                u->stride[2], u->stride[1]);
    }
    // Wide B: B B^T = W diag(S^2) W^T
    if ((rc = run_gram(C, z, P.n, P.n4, g))) return rc;
    const size_t eig_smem = static_cast<size_t>(2) * (P.k + (P.k & 1)) * (P.k + (P.k & 1) + 1) * 8;
    eig_kernel<<<static_cast<unsigned>(P.batch), kEigThreads, eig_smem, strm>>>(
        g, P.k, rank, static_cast<float*>(s->data), s->stride[0], s->stride[1], mu, mv, 30);
    if (cudaGetLastError() != cudaSuccess) return fail_msg(ADA_ERR_LAUNCH, "eigen-solve launch failed");
    // U = Q W[:, :r]; Vh = diag(1/S) W[:, :r]^T B  (low_rank.py:102-107)
    if ((rc = run_apply<float>(C, y, P.m, P.m4, mu, rank, 0, static_cast<float*>(u->data), u->stride[0],
                               u->stride[2], u->stride[1])))
        return rc;
    if ((rc = run_apply<float>(C, z, P.n, P.n4, mv, rank, 0, static_cast<float*>(vh->data), vh->stride[0],
                               vh->stride[1], vh->stride[2])))
        return rc;
    return ADA_OK;
}
