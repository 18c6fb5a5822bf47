// K3 operand step: the low-rank projection q_low = q W^T, k_low = k W^T on the
// sm_100a tensor cores (src/adaattn/attention/adaattn.py:357-358, where
// rank_proj_down is a bias-free Linear(D -> r) applied in the inputs' dtype).
//
// Persistent CTAs walk work items (one item = 128 rows of q or of k of one
// (b, h) slice whose decision is the low-rank branch). Per item a TMA load
// brings the 128 x D tile, one tcgen05 MMA chain computes the 128 x r block
// with fp32 accumulation in tensor memory, and the epilogue rounds it to the
// inputs' dtype (the reference's Linear returns that dtype) and stores it in
// the head's compute format: fp16/bf16 into the 16-bit operand region (zero
// padded to r_pad columns) or fp32 into the fp32 region. W is loaded once per
// CTA. Warp roles (256 threads): warp 0 TMA, warp 1 TMEM + MMA issue, warps
// 4-7 epilogue (one row per thread); warps 2-3 idle.
#include "ada_common.cuh"
#include "ada_internal.h"

namespace ada {
namespace {

constexpr int kProjThreads = 256;
constexpr int kProjStages = 4;
constexpr int kStageBytes = 32 * 1024;  // one staged 128 x 64 output tile (fp32)

struct __align__(8) ProjBarriers {
    uint64_t w_full;
    uint64_t x_full[kProjStages];
    uint64_t x_empty[kProjStages];
    uint64_t acc_full[2];
    uint64_t acc_empty[2];
    uint64_t teardown;
    uint32_t tmem_base;
    int abort_flag;
};

struct ProjItem {
    int64_t bh;
    int which;  // 0: q, 1: k
    int tile;
};

__device__ __forceinline__ bool proj_item(const ProjLaunch& L, int64_t it, int ntq, int ntk, ProjItem* w,
                                          int* prec) {
    const int per = ntq + ntk;
    w->bh = it / per;
    const int rem = static_cast<int>(it % per);
    w->which = rem < ntq ? 0 : 1;
    w->tile = rem < ntq ? rem : rem - ntq;
    int low;
    get_decision(L.dec, w->bh, prec, &low);
    return low && (((L.tc16_mask | L.fp32_mask | L.in16_mask) >> *prec) & 1u);
}

template <int D, int RP>
__global__ void __launch_bounds__(kProjThreads, 1) proj_tc_kernel(const __grid_constant__ ProjLaunch L) {
    constexpr int ATOMS = D / 64;           // 64 16-bit elements per 128-byte row
    constexpr int BOX = 128 * 128;          // one 128-row x 128-byte box
    constexpr int X_BYTES = 128 * D * 2;
    constexpr int W_BYTES = RP * D * 2;
    constexpr int W_BOX = RP * 128;
    constexpr uint32_t IDESC = make_idesc(0, 0, 0, 0, 128, RP);  // format bits patched below
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sW = base;
    uint8_t* sX = base + W_BYTES;
    uint8_t* sStage = sX + kProjStages * X_BYTES;  // [2][32 KB] output staging (RP 64)
    ProjBarriers* bars = reinterpret_cast<ProjBarriers*>(sStage + (RP == 64 ? 2 * kStageBytes : 0));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t fmt = L.in_dtype == ADA_BF16 ? 1u : 0u;
    const uint32_t idesc = IDESC | (fmt << 7) | (fmt << 10);

    const int ntq = static_cast<int>((L.Nq + 127) / 128);
    const int ntk = static_cast<int>((L.Nk + 127) / 128);
    const int64_t n_items = L.B * L.H * (ntq + ntk);

    // No low-rank head in this launch's precisions: nothing to project.
    {
        int any = 0;
        for (int64_t bh = threadIdx.x; bh < L.B * L.H && !any; bh += blockDim.x) {
            int prec, low;
            get_decision(L.dec, bh, &prec, &low);
            any = low && (((L.tc16_mask | L.fp32_mask | L.in16_mask) >> prec) & 1u);
        }
        if (!__syncthreads_or(any)) return;
    }

    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&bars->w_full), 1);
        for (int s = 0; s < kProjStages; ++s) {
            mbar_init(smem_u32(&bars->x_full[s]), 1);
            mbar_init(smem_u32(&bars->x_empty[s]), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(smem_u32(&bars->acc_full[a]), 1);
            mbar_init(smem_u32(&bars->acc_empty[a]), 128);
        }
        mbar_init(smem_u32(&bars->teardown), 1);
        bars->abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(&bars->tmem_base), 256);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;
    volatile int* abort_flag = &bars->abort_flag;
    const uint64_t tmo = L.timeout_ns;

    if (warp == 0) {
        if (lane == 0) {
            tma_prefetch_desc(&L.tq);
            tma_prefetch_desc(&L.tk);
            const uint32_t wbar = smem_u32(&bars->w_full);
            mbar_arrive_expect_tx(wbar, W_BYTES);
            for (int a = 0; a < ATOMS; ++a) tma_load_2d(smem_u32(sW + a * W_BOX), &L.tw, wbar, a * 64, 0);
            uint32_t xi = 0;
            bool ok = true;
            for (int64_t it = blockIdx.x; ok && it < n_items; it += gridDim.x) {
                ProjItem w;
                int prec;
                if (!proj_item(L, it, ntq, ntk, &w, &prec)) continue;
                const uint32_t st = xi % kProjStages;
                ok = mbar_wait(smem_u32(&bars->x_empty[st]), ((xi / kProjStages) & 1u) ^ 1u, abort_flag, tmo,
                               L.status);
                if (!ok) break;
                const uint32_t fbar = smem_u32(&bars->x_full[st]);
                mbar_arrive_expect_tx(fbar, X_BYTES);
                const int b = static_cast<int>(w.bh / L.H), h = static_cast<int>(w.bh % L.H);
                const CUtensorMap* map = w.which == 0 ? &L.tq : &L.tk;
                for (int a = 0; a < ATOMS; ++a)
                    tma_load_4d(smem_u32(sX + st * X_BYTES + a * BOX), map, fbar, a * 64, w.tile * 128, h, b);
                ++xi;
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            bool ok = mbar_wait(smem_u32(&bars->w_full), 0, abort_flag, tmo, L.status);
            uint32_t xi = 0;
            for (int64_t it = blockIdx.x; ok && it < n_items; it += gridDim.x) {
                ProjItem w;
                int prec;
                if (!proj_item(L, it, ntq, ntk, &w, &prec)) continue;
                const uint32_t st = xi % kProjStages;
                const uint32_t ab = xi & 1u;
                ok = mbar_wait(smem_u32(&bars->acc_empty[ab]), ((xi >> 1) & 1u) ^ 1u, abort_flag, tmo, L.status);
                if (!ok) break;
                ok = mbar_wait(smem_u32(&bars->x_full[st]), (xi / kProjStages) & 1u, abort_flag, tmo, L.status);
                if (!ok) break;
                tc_fence_after();
                const uint32_t x0 = smem_u32(sX + st * X_BYTES);
                const uint32_t w0 = smem_u32(sW);
#pragma unroll
                for (int ks = 0; ks < D / 16; ++ks) {
                    const uint32_t off = (ks / 4) * BOX + (ks % 4) * 32;
                    const uint32_t woff = (ks / 4) * W_BOX + (ks % 4) * 32;
                    mma_ss_f16(tmem + ab * 128, make_sdesc_sw128(x0 + off, 16, 1024),
                               make_sdesc_sw128(w0 + woff, 16, 1024), idesc, ks > 0 ? 1u : 0u);
                }
                tc_commit(smem_u32(&bars->x_empty[st]));
                tc_commit(smem_u32(&bars->acc_full[ab]));
                ++xi;
            }
            tc_commit(smem_u32(&bars->teardown));
            // bounded wait for the last products before the CTA frees TMEM
            const uint64_t t0 = globaltimer_ns();
            uint32_t spins = 0;
            while (!mbar_try_wait(smem_u32(&bars->teardown), 0)) {
                if ((++spins & 63u) == 0u && globaltimer_ns() - t0 > tmo) {
                    record_error(L.status, ADA_ERR_TIMEOUT);
                    break;
                }
            }
        }
        __syncwarp();
    } else if (warp >= 4) {
        const int r_reg = L.r, in_dtype_reg = L.in_dtype;
        const int row = (warp & 3) * 32 + lane;
        const uint32_t lane_bits = static_cast<uint32_t>((warp & 3) * 32) << 16;
        const bool leader = threadIdx.x == 128;
        uint32_t xi = 0;
        bool ok = true;
        for (int64_t it = blockIdx.x; ok && it < n_items; it += gridDim.x) {
            ProjItem w;
            int prec;
            if (!proj_item(L, it, ntq, ntk, &w, &prec)) continue;
            const uint32_t ab = xi & 1u;
            ok = mbar_wait(smem_u32(&bars->acc_full[ab]), (xi >> 1) & 1u, abort_flag, tmo, L.status);
            if (!ok) break;
            tc_fence_after();
            float y[RP];
#pragma unroll
            for (int c = 0; c < RP / 32; ++c) {
                uint32_t r[32];
                tmem_ld32(tmem + lane_bits + ab * 128 + c * 32, r);
                tmem_ld_wait();
                reg_fence32(r);
#pragma unroll
                for (int i = 0; i < 32; ++i) y[c * 32 + i] = __uint_as_float(r[i]);
            }
            tc_fence_before();
            mbar_arrive(smem_u32(&bars->acc_empty[ab]));
            const uint32_t item_no = xi++;
            const int64_t nrows = w.which == 0 ? L.Nq : L.Nk;
            const int64_t grow = static_cast<int64_t>(w.tile) * 128 + row;
            // The reference's Linear returns the inputs' dtype. (Launch
            // fields are copied to registers first: the asm memory clobbers
            // above would otherwise make the loop reload them each step.)
            const int rr = r_reg, in_dt = in_dtype_reg;
#pragma unroll
            for (int i = 0; i < RP; ++i) y[i] = i < rr ? round_to(y[i], in_dt) : 0.f;
            const bool to32 = (L.fp32_mask >> prec) & 1u;
            // E4M3 heads keep q_low/k_low in the inputs' dtype for the quantiser.
            const bool f16 = ((L.in16_mask >> prec) & 1u) ? (in_dt == ADA_F16) : ((L.f16_mask >> prec) & 1u);
            if constexpr (RP == 64) {
                if (to32 ? L.tma32 : L.tma16) {
                    // Stage the 128-row tile in the swizzled box layout and let
                    // one thread store it with TMA (rows past N are clipped).
                    uint8_t* stg = sStage + (item_no & 1u) * kStageBytes;
                    if (leader) bulk_wait_group_read1();  // the store from this buffer two items ago
                    named_barrier_sync(1, 128);
                    if (to32) {
#pragma unroll
                        for (int k = 0; k < 2; ++k) {
                            uint8_t* line = stg + k * (128 * 128) + row * 128;
#pragma unroll
                            for (int c = 0; c < 8; ++c)
                                *reinterpret_cast<float4*>(line + ((c ^ (row & 7)) * 16)) =
                                    make_float4(y[k * 32 + 4 * c], y[k * 32 + 4 * c + 1], y[k * 32 + 4 * c + 2],
                                                y[k * 32 + 4 * c + 3]);
                        }
                    } else {
                        uint8_t* line = stg + row * 128;
#pragma unroll
                        for (int c = 0; c < 8; ++c) {
                            uint32_t p[4];
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const float lo = y[8 * c + 2 * e], hi = y[8 * c + 2 * e + 1];
                                p[e] = f16 ? pack_f16x2(lo, hi) : pack_bf16x2(lo, hi);
                            }
                            *reinterpret_cast<uint4*>(line + ((c ^ (row & 7)) * 16)) = make_uint4(p[0], p[1], p[2], p[3]);
                        }
                    }
                    fence_proxy_async_smem();
                    named_barrier_sync(1, 128);
                    if (leader) {
                        const int bh = static_cast<int>(w.bh);
                        if (to32) {
                            const CUtensorMap* map = w.which == 0 ? &L.to32_q : &L.to32_k;
                            for (int k = 0; k < 2 && k * 32 < L.r; ++k)
                                tma_store_3d(map, smem_u32(stg + k * (128 * 128)), k * 32, w.tile * 128, bh);
                        } else {
                            tma_store_3d(w.which == 0 ? &L.to16_q : &L.to16_k, smem_u32(stg), 0, w.tile * 128, bh);
                        }
                        bulk_commit_group();
                    }
                    continue;
                }
            }
            if (grow >= nrows) continue;
            if (to32) {
                float* out = (w.which == 0 ? L.ws32_q : L.ws32_k) + (w.bh * nrows + grow) * L.r;
#pragma unroll
                for (int i = 0; i < RP; ++i)
                    if (i < L.r) out[i] = y[i];
            } else {
                uint16_t* out = reinterpret_cast<uint16_t*>(w.which == 0 ? L.ws16_q : L.ws16_k) +
                                (w.bh * nrows + grow) * L.ld16;
                uint4* dst = reinterpret_cast<uint4*>(out);
#pragma unroll
                for (int v = 0; v < RP / 8; ++v) {
                    uint32_t p[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float lo = y[v * 8 + 2 * e], hi = y[v * 8 + 2 * e + 1];
                        p[e] = f16 ? pack_f16x2(lo, hi) : pack_bf16x2(lo, hi);
                    }
                    dst[v] = make_uint4(p[0], p[1], p[2], p[3]);
                }
            }
        }
        if (leader) bulk_wait_group0();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 256);
    }
}

template <int D, int RP>
int launch_proj(const ProjLaunch& L, cudaStream_t stream) {
    constexpr int smem = RP * D * 2 + kProjStages * 128 * D * 2 + (RP == 64 ? 2 * kStageBytes : 0) + 1024 + 256;
    auto kern = proj_tc_kernel<D, RP>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
        return ADA_ERR_LAUNCH;
    const int64_t items = L.B * L.H * ((L.Nq + 127) / 128 + (L.Nk + 127) / 128);
    if (items <= 0) return ADA_OK;
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
        return ADA_ERR_LAUNCH;
    const int64_t grid = items < sms ? items : sms;
    kern<<<static_cast<unsigned>(grid), kProjThreads, smem, stream>>>(L);
    return cudaGetLastError() == cudaSuccess ? ADA_OK : ADA_ERR_LAUNCH;
}

}  // namespace

int launch_proj_tc(const ProjLaunch& L, cudaStream_t stream) {
    if (L.D == 128 && L.r_pad == 64) return launch_proj<128, 64>(L, stream);
    if (L.D == 128 && L.r_pad == 128) return launch_proj<128, 128>(L, stream);
    if (L.D == 64 && L.r_pad == 64) return launch_proj<64, 64>(L, stream);
    return ADA_ERR_UNSUPPORTED;
}

}  // namespace ada
