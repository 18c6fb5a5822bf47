// K1: the runtime analyzer. One CTA per (b, h) computes the statistics of the
// sampled score block, then one CTA turns them into decisions, per head or
// for the whole call. Restates src/adaattn/attention/adaattn.py:246-289.
//
// Every intermediate is rounded to the inputs' dtype exactly where the
// reference's PyTorch ops produce a tensor of that dtype (matmul output,
// scaled scores, softmax output, p + eps, log, p * log, row sums, the
// normalised entropy and its mean), so decisions agree with the reference
// except where a statistic sits within rounding distance of a threshold.
#include "ada_common.cuh"
#include "ada_internal.h"

namespace ada {

namespace {

constexpr int kSample = 64;
constexpr int kThreads = 256;

struct StatsArgs {
    const void* q;
    const void* k;
    int dtype;
    int64_t B, H, Nq, Nk, D;
    int64_t qs[4], ks[4];
    float scale, eps, log_s;
    int S, stride;
    int vec;            // 16-bit q and k with unit column stride and 16-byte aligned rows, D % 8 == 0
    float* head_stats;  // [B*H*4]
    float* head_sum;    // [B*H]  sum over sampled rows of the normalised row entropy
};

// Per-row softmax, entropy and maxima of the 64 x 64 raw sample scores `ss`
// ([64][65] in shared memory), then the head's statistics; every thread of
// the CTA (256) calls it. Scores are rounded the way the reference's ops
// round them (adaattn.py:256-275).
__device__ __forceinline__ void sample_stats(const float* ss, const StatsArgs& a, int bh, float* s_rows,
                                             unsigned int* s_max_score, unsigned int* s_max_prob) {
    const int tid = threadIdx.x;
    const int S = a.S;
    // Thread layout: 4 consecutive lanes own one sample row, 16 columns each.
    const int r = tid >> 2;
    const int c0 = (tid & 3) * 16;
    const bool row_ok = r < S;
    float sc[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) sc[j] = ss[r * (kSample + 1) + c0 + j];
    // scores = round(round(q k^T) * scale); track max |score|.
    float local_max_abs = 0.f;
    float row_max = -INFINITY;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const bool ok = row_ok && (c0 + j) < S;
        float s = round_to(round_to(sc[j], a.dtype) * a.scale, a.dtype);
        sc[j] = ok ? s : -INFINITY;
        if (ok) {
            local_max_abs = fmaxf(local_max_abs, fabsf(s));
            row_max = fmaxf(row_max, s);
        }
    }
    row_max = fmaxf(row_max, __shfl_xor_sync(0xffffffffu, row_max, 1));
    row_max = fmaxf(row_max, __shfl_xor_sync(0xffffffffu, row_max, 2));
    // softmax in fp32 on the rounded scores, output rounded to the dtype.
    float e[16];
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        e[j] = (sc[j] == -INFINITY) ? 0.f : expf(sc[j] - row_max);
        sum += e[j];
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    const float inv = 1.f / sum;
    float local_max_prob = 0.f;
    float ent = 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        if (row_ok && (c0 + j) < S) {
            const float p = round_to(e[j] * inv, a.dtype);
            local_max_prob = fmaxf(local_max_prob, p);
            const float t1 = round_to(p + a.eps, a.dtype);
            const float t2 = round_to(logf(t1), a.dtype);
            ent += round_to(p * t2, a.dtype);
        }
    }
    ent += __shfl_xor_sync(0xffffffffu, ent, 1);
    ent += __shfl_xor_sync(0xffffffffu, ent, 2);
    if (row_ok && (tid & 3) == 0) {
        const float row_entropy = -round_to(ent, a.dtype);
        s_rows[r] = round_to(row_entropy / a.log_s, a.dtype);
    }
    // block maxima (non-negative floats compare like their bit patterns)
    for (int o = 16; o > 0; o >>= 1) {
        local_max_abs = fmaxf(local_max_abs, __shfl_xor_sync(0xffffffffu, local_max_abs, o));
        local_max_prob = fmaxf(local_max_prob, __shfl_xor_sync(0xffffffffu, local_max_prob, o));
    }
    __syncthreads();
    if ((tid & 31) == 0) {
        atomicMax(s_max_score, __float_as_uint(local_max_abs));
        atomicMax(s_max_prob, __float_as_uint(local_max_prob));
    }
    __syncthreads();
    if (tid < 32) {
        float v = 0.f;
        for (int i = tid; i < S; i += 32) v += s_rows[i];
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (tid == 0) {
            const float ne = round_to(v / static_cast<float>(S), a.dtype);
            float* hs = a.head_stats + static_cast<int64_t>(bh) * 4;
            hs[0] = ne;
            hs[1] = __uint_as_float(*s_max_score);
            hs[2] = __uint_as_float(*s_max_prob);
            hs[3] = ne * static_cast<float>(a.Nq < a.Nk ? a.Nq : a.Nk);
            a.head_sum[bh] = v;
        }
    }
}

__global__ void __launch_bounds__(kThreads) analyze_stats_kernel(StatsArgs a) {
    extern __shared__ __align__(16) float sm[];
    const int D = static_cast<int>(a.D);
    const int DP = (D + 3) & ~3;  // columns D..DP-1 hold zeros
    const int ld = DP + 4;        // 16-byte rows, staggered banks
    float* sq = sm;
    float* sk = sm + kSample * ld;
    float* ss = sk + kSample * ld;  // [kSample][kSample + 1] raw scores
    __shared__ unsigned int s_max_score, s_max_prob;
    __shared__ float s_rows[kSample];

    const int bh = blockIdx.x;
    const int b = bh / static_cast<int>(a.H);
    const int h = bh % static_cast<int>(a.H);
    const int tid = threadIdx.x;
    const int S = a.S;
    if (tid == 0) {
        s_max_score = 0u;
        s_max_prob = 0u;
    }
    const int64_t qbase = b * a.qs[0] + h * a.qs[1];
    const int64_t kbase = b * a.ks[0] + h * a.ks[1];
    if (a.vec) {
        // 16-byte loads in rounds of 4 per thread and tensor, all of a round
        // in flight before the first use (S * D / 8 groups: one round up to
        // D = 128, two at D = 256).
        const int g = D >> 3;
        const int n = S * g;
        for (int base = 0; base < n; base += 4 * kThreads) {
            uint4 vq[4], vk[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int idx = base + tid + u * kThreads;
                if (idx < n) {
                    const int r = idx / g, c = (idx - r * g) * 8;
                    const int64_t row = static_cast<int64_t>(r) * a.stride;
                    vq[u] = reinterpret_cast<const uint4*>(a.q)[(qbase + row * a.qs[2] + c) / 8];
                    vk[u] = reinterpret_cast<const uint4*>(a.k)[(kbase + row * a.ks[2] + c) / 8];
                }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int idx = base + tid + u * kThreads;
                if (idx < n) {
                    const int r = idx / g, c = (idx - r * g) * 8;
                    const uint32_t wq[4] = {vq[u].x, vq[u].y, vq[u].z, vq[u].w};
                    const uint32_t wk[4] = {vk[u].x, vk[u].y, vk[u].z, vk[u].w};
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        float q0, q1, k0, k1;
                        if (a.dtype == ADA_BF16) {
                            q0 = __uint_as_float(wq[i] << 16);
                            q1 = __uint_as_float(wq[i] & 0xffff0000u);
                            k0 = __uint_as_float(wk[i] << 16);
                            k1 = __uint_as_float(wk[i] & 0xffff0000u);
                        } else {
                            unpack_f16x2(wq[i], q0, q1);
                            unpack_f16x2(wk[i], k0, k1);
                        }
                        sq[r * ld + c + 2 * i] = q0;
                        sq[r * ld + c + 2 * i + 1] = q1;
                        sk[r * ld + c + 2 * i] = k0;
                        sk[r * ld + c + 2 * i + 1] = k1;
                    }
                }
            }
        }
    } else {
        for (int idx = tid; idx < S * D; idx += kThreads) {
            const int r = idx / D, d = idx - r * D;
            const int64_t row = static_cast<int64_t>(r) * a.stride;
            sq[r * ld + d] = load_as_f32(a.q, qbase + row * a.qs[2] + d * a.qs[3], a.dtype);
            sk[r * ld + d] = load_as_f32(a.k, kbase + row * a.ks[2] + d * a.ks[3], a.dtype);
        }
    }
    for (int idx = tid; idx < S * (DP - D); idx += kThreads) {
        const int r = idx / (DP - D), d = D + idx - r * (DP - D);
        sq[r * ld + d] = 0.f;
        sk[r * ld + d] = 0.f;
    }
    __syncthreads();
    // q k^T of the sample: each thread a 4 x 4 block (rows 4*ty + i, columns
    // tx + 16*j), 16-byte shared loads; every score is one fma chain over
    // d = 0, 1, ..., D-1 (the zero padding adds nothing).
    {
        const int ty = tid >> 4, tx = tid & 15;
        float acc[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
        for (int d = 0; d < DP; d += 4) {
            float4 qa[4], kb[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) qa[i] = *reinterpret_cast<const float4*>(sq + (ty * 4 + i) * ld + d);
#pragma unroll
            for (int j = 0; j < 4; ++j) kb[j] = *reinterpret_cast<const float4*>(sk + (tx + 16 * j) * ld + d);
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    acc[i][j] = fmaf(qa[i].x, kb[j].x, acc[i][j]);
                    acc[i][j] = fmaf(qa[i].y, kb[j].y, acc[i][j]);
                    acc[i][j] = fmaf(qa[i].z, kb[j].z, acc[i][j]);
                    acc[i][j] = fmaf(qa[i].w, kb[j].w, acc[i][j]);
                }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) ss[(ty * 4 + i) * (kSample + 1) + tx + 16 * j] = acc[i][j];
    }
    __syncthreads();

    sample_stats(ss, a, bh, s_rows, &s_max_score, &s_max_prob);
}


// The same statistics with the 64 x 64 x D sample product on the tensor
// cores, for 16-bit q, k whose rows are 16-byte aligned and D % 16 == 0
// (D <= 256). The sample rows are written to shared memory in the 128-byte
// swizzled K-major layout (q as a 128-row A operand whose rows 64..127 are
// zero, k as a 64-row B operand); one thread issues D / 16 tcgen05.mma
// (M = 128, N = 64, fp32 accumulate) into 64 TMEM columns and commits to an
// mbarrier (bounded wait); warps 0 and 1 then read their 32 rows each and
// run the per-row softmax and entropy with the reference's roundings, one
// row per thread. The products are exact and summed in fp32, as in the
// CUDA-core kernel (the order of the sum differs).
struct StatsTcArgs {
    StatsArgs a;
    unsigned int* status;
    uint64_t timeout_ns;
};

__global__ void __launch_bounds__(kThreads) analyze_stats_tc_kernel(const __grid_constant__ StatsTcArgs T) {
    const StatsArgs& a = T.a;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int D = static_cast<int>(a.D);
    const int boxes = (D + 63) / 64;
    uint8_t* sA = base;                        // boxes x [128 rows x 128 B]
    uint8_t* sB = base + boxes * 128 * 128;    // boxes x [64 rows x 128 B]
    float* ss = reinterpret_cast<float*>(sA);  // [64][65] raw scores, over A once the product is done
    __shared__ __align__(8) uint64_t bar;
    __shared__ uint32_t tmem_base;
    __shared__ int abort_flag;
    __shared__ unsigned int s_max_score, s_max_prob;
    __shared__ float s_rows[kSample];
    const int bh = blockIdx.x;
    const int b = bh / static_cast<int>(a.H);
    const int h = bh % static_cast<int>(a.H);
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int S = a.S;
    if (tid == 0) {
        mbar_init(smem_u32(&bar), 1);
        abort_flag = 0;
        s_max_score = 0u;
        s_max_prob = 0u;
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(smem_u32(&tmem_base), 64);
        tmem_relinquish();
    }
    // Sample rows -> swizzled tiles: 16-byte chunk c of row r goes to chunk
    // (c & 7) ^ (r & 7) of that row's 128-byte line in box c / 8. A thread's
    // loads (at most 8 per tensor at D = 256) are all in flight before the
    // first store.
    const int64_t qbase = b * a.qs[0] + h * a.qs[1];
    const int64_t kbase = b * a.ks[0] + h * a.ks[1];
    const int g = D >> 3;  // 16-byte chunks per row
    const int n = kSample * g;
    constexpr int kMaxPer = (kSample * 32 + kThreads - 1) / kThreads;  // D <= 256
    uint4 vq[kMaxPer], vk[kMaxPer];
#pragma unroll
    for (int u = 0; u < kMaxPer; ++u) {
        const int idx = tid + u * kThreads;
        vq[u] = make_uint4(0u, 0u, 0u, 0u);
        vk[u] = vq[u];
        if (idx < n) {
            const int r = idx / g, c = idx - r * g;
            if (r < S) {
                const int64_t row = static_cast<int64_t>(r) * a.stride;
                vq[u] = reinterpret_cast<const uint4*>(a.q)[(qbase + row * a.qs[2] + c * 8) / 8];
                vk[u] = reinterpret_cast<const uint4*>(a.k)[(kbase + row * a.ks[2] + c * 8) / 8];
            }
        }
    }
#pragma unroll
    for (int u = 0; u < kMaxPer; ++u) {
        const int idx = tid + u * kThreads;
        if (idx < n) {
            const int r = idx / g, c = idx - r * g;
            const int off = r * 128 + (((c & 7) ^ (r & 7)) << 4);
            *reinterpret_cast<uint4*>(sA + (c >> 3) * (128 * 128) + off) = vq[u];
            *reinterpret_cast<uint4*>(sB + (c >> 3) * (64 * 128) + off) = vk[u];
        }
    }
    // rows 64..127 of the A operand: zero
    for (int idx = tid; idx < n; idx += kThreads) {
        const int r = kSample + idx / g, c = idx % g;
        *reinterpret_cast<uint4*>(sA + (c >> 3) * (128 * 128) + r * 128 + (((c & 7) ^ (r & 7)) << 4)) =
            make_uint4(0u, 0u, 0u, 0u);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;
    if (tid == 0) {
        const uint32_t fmt = a.dtype == ADA_BF16 ? 1u : 0u;
        const uint32_t idesc = make_idesc(fmt, fmt, 0, 0, 128, 64);
        const uint32_t a0 = smem_u32(sA), b0 = smem_u32(sB);
        for (int ks = 0; ks < D / 16; ++ks) {
            const uint32_t box = static_cast<uint32_t>(ks >> 2), inner = static_cast<uint32_t>((ks & 3) * 32);
            mma_ss_f16(tmem, make_sdesc_sw128(a0 + box * (128 * 128) + inner, 16, 1024),
                       make_sdesc_sw128(b0 + box * (64 * 128) + inner, 16, 1024), idesc, ks > 0 ? 1u : 0u);
        }
        tc_commit(smem_u32(&bar));
    }
    const bool ok = mbar_wait(smem_u32(&bar), 0, &abort_flag, T.timeout_ns, T.status);
    tc_fence_after();
    // every MMA has completed (or the wait gave up): A may be overwritten
    if (warp < 2) {
        const int r = warp * 32 + lane;  // TMEM lane == sample row
        uint32_t u0[32], u1[32];
        const uint32_t taddr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
        tmem_ld32(taddr, u0);
        tmem_ld32(taddr + 32, u1);
        tmem_ld_wait();
        reg_fence32(u0);
        reg_fence32(u1);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            ss[r * (kSample + 1) + j] = ok ? __uint_as_float(u0[j]) : NAN;
            ss[r * (kSample + 1) + 32 + j] = ok ? __uint_as_float(u1[j]) : NAN;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 64);
    }
    sample_stats(ss, a, bh, s_rows, &s_max_score, &s_max_prob);
}

struct DecideArgs {
    const float* head_stats;
    const float* head_sum;
    int32_t* decisions;
    float* summary;
    int64_t BH;
    int S;
    int dtype;
    int64_t min_n;
    double rank_threshold;
    int enable_rank, enable_prec, default_prec, allow_fp8, granularity;
};

__device__ __forceinline__ void decide_one(double ne, double ms, double mp, const DecideArgs& a,
                                           int* prec, int* low) {
    // adaattn.py:268-287, compared in double as the reference's Python floats are.
    *low = (a.enable_rank && ne < a.rank_threshold) ? 1 : 0;
    int p;
    if (ms > 50.0 || mp > 0.95)
        p = ADA_PREC_FP32;
    else if (ne > 0.8)
        p = a.allow_fp8 ? ADA_PREC_FP8 : ADA_PREC_FP16;
    else if (ne < 0.3)
        p = ADA_PREC_BF16;
    else
        p = a.default_prec;
    if (!a.enable_prec) p = a.default_prec;
    *prec = p;
}

__device__ __forceinline__ int prec_slot(int p) {
    // _precision_distribution index; AUTO falls in slot 0 (.get(precision, 0)).
    return (p >= ADA_PREC_FP32 && p <= ADA_PREC_FP8) ? p : 0;
}

__global__ void __launch_bounds__(kThreads) decide_kernel(DecideArgs a) {
    __shared__ float s_sum[kThreads / 32];
    __shared__ unsigned int s_ms, s_mp;
    __shared__ int s_cnt[5];
    const int tid = threadIdx.x;
    if (tid < 5) s_cnt[tid] = 0;
    if (tid == 0) {
        s_ms = 0u;
        s_mp = 0u;
    }
    __syncthreads();
    if (a.granularity == 0) {
        for (int64_t i = tid; i < a.BH; i += kThreads) {
            const float* hs = a.head_stats + i * 4;
            int p, low;
            decide_one(hs[0], hs[1], hs[2], a, &p, &low);
            a.decisions[i * 2 + 0] = p;
            a.decisions[i * 2 + 1] = low;
            atomicAdd(&s_cnt[prec_slot(p)], 1);
            if (low) atomicAdd(&s_cnt[4], 1);
        }
        __syncthreads();
        if (tid == 0) {
            a.summary[ADA_SUM_NE] = NAN;
            a.summary[ADA_SUM_MAX_SCORE] = NAN;
            a.summary[ADA_SUM_MAX_PROB] = NAN;
            a.summary[ADA_SUM_EFF_RANK] = NAN;
            a.summary[ADA_SUM_N_LOWRANK] = static_cast<float>(s_cnt[4]);
            for (int i = 0; i < 4; ++i) a.summary[ADA_SUM_N_FP32 + i] = static_cast<float>(s_cnt[i]);
            a.summary[ADA_SUM_N_TOTAL] = static_cast<float>(a.BH);
        }
        return;
    }
    // One decision for the whole call: mean of every sampled row's normalised
    // entropy over all heads, maxima over all heads.
    float v = 0.f, ms = 0.f, mp = 0.f;
    for (int64_t i = tid; i < a.BH; i += kThreads) {
        v += a.head_sum[i];
        ms = fmaxf(ms, a.head_stats[i * 4 + 1]);
        mp = fmaxf(mp, a.head_stats[i * 4 + 2]);
    }
    for (int o = 16; o > 0; o >>= 1) {
        v += __shfl_xor_sync(0xffffffffu, v, o);
        ms = fmaxf(ms, __shfl_xor_sync(0xffffffffu, ms, o));
        mp = fmaxf(mp, __shfl_xor_sync(0xffffffffu, mp, o));
    }
    if ((tid & 31) == 0) {
        s_sum[tid >> 5] = v;
        atomicMax(&s_ms, __float_as_uint(ms));
        atomicMax(&s_mp, __float_as_uint(mp));
    }
    __syncthreads();
    __shared__ int s_dec[2];
    __shared__ float s_ne;
    if (tid == 0) {
        float tot = 0.f;
        for (int i = 0; i < kThreads / 32; ++i) tot += s_sum[i];
        const float ne =
            round_to(tot / static_cast<float>(static_cast<double>(a.BH) * a.S), a.dtype);
        int p, low;
        decide_one(ne, __uint_as_float(s_ms), __uint_as_float(s_mp), a, &p, &low);
        s_dec[0] = p;
        s_dec[1] = low;
        s_ne = ne;
        a.summary[ADA_SUM_NE] = ne;
        a.summary[ADA_SUM_MAX_SCORE] = __uint_as_float(s_ms);
        a.summary[ADA_SUM_MAX_PROB] = __uint_as_float(s_mp);
        a.summary[ADA_SUM_EFF_RANK] = ne * static_cast<float>(a.min_n);
        a.summary[ADA_SUM_N_LOWRANK] = static_cast<float>(low);
        for (int i = 0; i < 4; ++i) a.summary[ADA_SUM_N_FP32 + i] = (prec_slot(p) == i) ? 1.f : 0.f;
        a.summary[ADA_SUM_N_TOTAL] = 1.f;
    }
    __syncthreads();
    for (int64_t i = tid; i < a.BH; i += kThreads) {
        a.decisions[i * 2 + 0] = s_dec[0];
        a.decisions[i * 2 + 1] = s_dec[1];
    }
}

// ---------------------------------------------------------------------------
// _adaattn_cuda helper ops (bindings.cpp:101-135) on the device.
// ---------------------------------------------------------------------------
struct EntropyArgs {
    const void* w;
    int dtype;
    int64_t rows, len;        // rows of length `len` (contiguous)
    int64_t group;            // >0: average `group` consecutive row entropies, then exp
    float* out;
};

// One warp per row: -sum w * log(w + 1e-10), each op rounded to the dtype.
__global__ void entropy_rows_kernel(EntropyArgs a) {
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= a.rows) return;
    const int64_t base = warp * a.len;
    float acc = 0.f;
    for (int64_t i = lane; i < a.len; i += 32) {
        const float w = load_as_f32(a.w, base + i, a.dtype);
        const float t = round_to(logf(round_to(w + 1e-10f, a.dtype)), a.dtype);
        acc += round_to(w * t, a.dtype);
    }
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) a.out[warp] = -round_to(acc, a.dtype);
}

// exp(mean over `group` consecutive rows of the row entropy): one warp per
// group walks its rows, so no intermediate buffer is needed.
__global__ void effective_rank_kernel(const void* w, int dtype, int64_t groups, int64_t group,
                                      int64_t len, float* out) {
    const int64_t g = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (g >= groups) return;
    float total = 0.f;
    for (int64_t row = 0; row < group; ++row) {
        const int64_t base = (g * group + row) * len;
        float acc = 0.f;
        for (int64_t i = lane; i < len; i += 32) {
            const float x = load_as_f32(w, base + i, dtype);
            const float t = round_to(logf(round_to(x + 1e-10f, dtype)), dtype);
            acc += round_to(x * t, dtype);
        }
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        total += -round_to(acc, dtype);
    }
    if (lane == 0) out[g] = round_to(expf(round_to(total / static_cast<float>(group), dtype)), dtype);
}

__global__ void target_ranks_kernel(const float* eff, int64_t n, int64_t min_rank, int64_t max_rank,
                                    double thr, int64_t* out) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float e = eff[i];
    if (static_cast<double>(e) < thr) {
        float v = e * 1.5f;
        v = fminf(fmaxf(v, static_cast<float>(min_rank)), static_cast<float>(max_rank));
        out[i] = static_cast<int64_t>(v);
    } else {
        out[i] = max_rank;
    }
}

// Waits on a barrier nothing signals; the bounded wait gives up and records
// ADA_ERR_TIMEOUT, after which the kernel returns normally.
__global__ void bounded_wait_kernel(uint64_t timeout_ns, unsigned int* status) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&bar), 1);
        abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) mbar_wait(smem_u32(&bar), 0, &abort_flag, timeout_ns, status);
    __syncthreads();
}

}  // namespace

int launch_analyze(const AnalyzeLaunch& L, cudaStream_t stream) {
    StatsArgs a{};
    a.q = L.q;
    a.k = L.k;
    a.dtype = L.dtype;
    a.B = L.B;
    a.H = L.H;
    a.Nq = L.Nq;
    a.Nk = L.Nk;
    a.D = L.D;
    for (int i = 0; i < 4; ++i) {
        a.qs[i] = L.qs[i];
        a.ks[i] = L.ks[i];
    }
    a.scale = L.scale;
    a.eps = L.eps;
    a.S = L.S;
    a.stride = L.stride;
    a.log_s = static_cast<float>(L.log_s);
    a.head_stats = L.head_stats;
    a.head_sum = L.head_sum;
    {
        auto rows16 = [](const void* p, const int64_t* st) {
            if (st[3] != 1 || (reinterpret_cast<uintptr_t>(p) & 15u) != 0) return false;
            for (int i = 0; i < 3; ++i)
                if (((st[i] * 2) % 16) != 0) return false;
            return true;
        };
        a.vec = (L.dtype == ADA_F16 || L.dtype == ADA_BF16) && (L.D % 8) == 0 && rows16(L.q, L.qs) &&
                rows16(L.k, L.ks);
    }
    if (a.vec && (L.D % 16) == 0 && L.D <= 256 && L.status != nullptr) {
        // tensor-core sample product: A 128 rows and B 64 rows per 64-column box
        const int boxes = static_cast<int>((L.D + 63) / 64);
        const size_t smem = static_cast<size_t>(boxes) * (128 + 64) * 128 + 1024;
        if (cudaFuncSetAttribute(analyze_stats_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem)) != cudaSuccess)
            return ADA_ERR_LAUNCH;
        StatsTcArgs t{};
        t.a = a;
        t.status = L.status;
        t.timeout_ns = L.timeout_ns;
        analyze_stats_tc_kernel<<<static_cast<unsigned>(L.B * L.H), kThreads, smem, stream>>>(t);
    } else {
        const size_t smem = static_cast<size_t>(2 * kSample * (((L.D + 3) & ~3) + 4) + kSample * (kSample + 1)) *
                            sizeof(float);
        if (smem > 48 * 1024) {
            if (cudaFuncSetAttribute(analyze_stats_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(smem)) != cudaSuccess)
                return ADA_ERR_LAUNCH;
        }
        analyze_stats_kernel<<<static_cast<unsigned>(L.B * L.H), kThreads, smem, stream>>>(a);
    }
    if (cudaGetLastError() != cudaSuccess) return ADA_ERR_LAUNCH;

    DecideArgs d{};
    d.head_stats = L.head_stats;
    d.head_sum = L.head_sum;
    d.decisions = L.decisions;
    d.summary = L.summary;
    d.BH = L.B * L.H;
    d.S = L.S;
    d.dtype = L.dtype;
    d.min_n = L.Nq < L.Nk ? L.Nq : L.Nk;
    d.rank_threshold = L.rank_threshold;
    d.enable_rank = L.enable_rank;
    d.enable_prec = L.enable_prec;
    d.default_prec = L.default_prec;
    d.allow_fp8 = L.allow_fp8;
    d.granularity = L.granularity;
    decide_kernel<<<1, kThreads, 0, stream>>>(d);
    return cudaGetLastError() == cudaSuccess ? ADA_OK : ADA_ERR_LAUNCH;
}

int launch_entropy_rows(const void* w, int dtype, int64_t rows, int64_t len, float* out,
                        cudaStream_t stream) {
    EntropyArgs a{w, dtype, rows, len, 0, out};
    const int threads = 256;
    const int64_t blocks = (rows * 32 + threads - 1) / threads;
    if (blocks > 0) entropy_rows_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(a);
    return cudaGetLastError() == cudaSuccess ? ADA_OK : ADA_ERR_LAUNCH;
}

int launch_effective_rank(const void* w, int dtype, int64_t groups, int64_t group, int64_t len,
                          float* out, cudaStream_t stream) {
    const int threads = 256;
    const int64_t blocks = (groups * 32 + threads - 1) / threads;
    if (blocks > 0)
        effective_rank_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(w, dtype, groups,
                                                                                    group, len, out);
    return cudaGetLastError() == cudaSuccess ? ADA_OK : ADA_ERR_LAUNCH;
}

int launch_target_ranks(const float* eff, int64_t n, int64_t min_rank, int64_t max_rank, double thr,
                        int64_t* out, cudaStream_t stream) {
    const int threads = 256;
    const int64_t blocks = (n + threads - 1) / threads;
    if (blocks > 0)
        target_ranks_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
            eff, n, min_rank, max_rank, thr, out);
    return cudaGetLastError() == cudaSuccess ? ADA_OK : ADA_ERR_LAUNCH;
}

int launch_bounded_wait(uint64_t timeout_ns, unsigned int* status, cudaStream_t stream) {
    bounded_wait_kernel<<<1, 32, 0, stream>>>(timeout_ns, status);
    return cudaGetLastError() == cudaSuccess ? ADA_OK : ADA_ERR_LAUNCH;
}

}  // namespace ada

// ---------------------------------------------------------------------------
// ada_analyze_noalloc: the analyzer without a caller-provided workspace.
//
// For callers that cannot call cudaMalloc -- for example code that must run
// inside a fixed device-memory budget set aside at start-up, or a caller whose
// memory allocator is not reachable from the place it runs the analyzer -- the
// per-head scratch that ada_analyze takes from the workspace lives here in a
// file-scope device array instead. Its size is fixed (kNoAllocMaxHeads floats,
// 256 KB), so batch * heads is limited to kNoAllocMaxHeads; every GPU that
// loads this library keeps the array until the process exits.
//
// Every call shares the one array: calls that overlap on the GPU (different
// streams, or different host threads on one device) race on it and must be
// ordered by the caller. Each call writes every scratch entry it reads
// before reading it, so nothing has to be cleared between calls.
//
// The first call on a device resolves the array's device address there
// (cudaGetSymbolAddress with that device current); make that first call
// before any stream capture. Nothing here calls cudaMalloc, cudaFree or an
// allocating library routine.
// ---------------------------------------------------------------------------
#include <cmath>
#include <mutex>

namespace ada {
namespace {

constexpr int64_t kNoAllocMaxHeads = 65536;
static __device__ __align__(256) float g_noalloc_head_sum[kNoAllocMaxHeads];

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[kNoAllocMaxDevices] = {nullptr};

// Once per device, with that device current (the caller has checked it is an
// sm_100 device): the device address of the array. In host code the array's
// name is only a host-side stand-in.
int noalloc_scratch(float** out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices)
        return record_last_error(ADA_ERR_DEVICE, "ada_analyze_noalloc: no usable current device");
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (g_noalloc_ptr[dev] == nullptr) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_head_sum);
        if (e != cudaSuccess || p == nullptr)
            return record_last_error(ADA_ERR_CUDA, "ada_analyze_noalloc: cudaGetSymbolAddress failed");
        g_noalloc_ptr[dev] = static_cast<float*>(p);
    }
    *out = g_noalloc_ptr[dev];
    return ADA_OK;
}

}  // namespace
}  // namespace ada

extern "C" int ada_analyze_noalloc(const AdaTensor* q, const AdaTensor* k, const AdaAnalyzeParams* params,
                                   int32_t* decisions, float* head_stats, float* summary, void* stream) {
    using namespace ada;
    AnalyzeLaunch L{};
    int rc = analyze_setup(q, k, params, decisions, head_stats, summary, &L);
    if (rc) return rc;
    // B * H > kNoAllocMaxHeads, tested without forming the product (no overflow)
    if (L.B > 0 && L.H > kNoAllocMaxHeads / L.B)
        return record_last_error(ADA_ERR_UNSUPPORTED,
                                 "ada_analyze_noalloc: batch * heads exceeds the fixed scratch of 65536 "
                                 "heads; use ada_analyze with a workspace");
    float* head_sum = nullptr;
    if ((rc = noalloc_scratch(&head_sum)) != ADA_OK) return rc;
    if (L.B * L.H == 0) return ADA_OK;
    L.head_sum = head_sum;
    if (launch_analyze(L, static_cast<cudaStream_t>(stream)) != ADA_OK)
        return record_last_error(ADA_ERR_LAUNCH, "ada_analyze_noalloc: launch failed");
    return ADA_OK;
}
