// The dense layers on either side of the attention path on the sm_100a tensor
// cores: y = act(x W^T + b) (+ r), the nn.Linear of the module's q/k/v
// projection and out_proj (src/adaattn/attention/adaattn.py:411-418 and :457)
// and of the transformer block that hosts it (its feed-forward and residual
// sums, examples/transformer_integration.py:33-58).
//
// x [M, K] and W [N, K] are 16-bit (both the same type), rows K-contiguous, so
// both operands are K-major. Persistent CTAs (one per SM) walk 128 x 256
// output tiles, M-fastest (the CTAs running together share one 256-row block
// of W, and x stays in L2). Per tile, 64-column K blocks of x (128 x 128 B)
// and W (256 x 128 B) stream through a 4-stage shared-memory ring filled by
// TMA; one thread issues 128 x 256 x 16 tcgen05 MMAs into an fp32
// accumulator in tensor memory. The accumulator is double buffered (2 x 256
// columns = all 512), so the epilogue of one tile overlaps the products of
// the next.
//
// Epilogue, per element, in the order the reference's PyTorch ops round:
//   t = round(acc + b)                   nn.Linear's output in the inputs' dtype
//   t = round(gelu(t))                   nn.GELU (erf form), when asked
//   t = round(t + r)                     the residual sum, when asked
// Warp roles (320 threads): warp 0 TMA producer, warp 1 TMEM allocation and
// MMA issue, warps 2-9 epilogue (warp w reads TMEM lanes 32 (w mod 4) .. +31,
// i.e. one output row per thread, and columns 128 ((w - 2) / 4) .. +127 of
// the tile). Every wait is bounded (ada::mbar_wait): a timeout raises the
// CTA's abort flag and ADA_ERR_TIMEOUT in the status word.
#include "ada_common.cuh"
#include "ada_internal.h"

namespace ada {
namespace {

constexpr int kLinThreads = 320;
constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 64;                       // 16-bit elements per 128-byte swizzle atom
constexpr int kStages = 4;
constexpr int kABytes = kBM * kBK * 2;        // 16 KB
constexpr int kBBytes = kBN * kBK * 2;        // 32 KB
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kStgBytes = 32 * 128;          // per epilogue warp: a 32-row x 64-column output tile
constexpr int kLinSmem = kStages * kStageBytes + 8 * kStgBytes + 1024 + 256;

struct __align__(8) LinBarriers {
    uint64_t full[kStages];
    uint64_t empty[kStages];
    uint64_t acc_full[2];
    uint64_t acc_empty[2];
    uint64_t teardown;
    uint64_t rfull[8];  // per epilogue warp: its residual tile has landed
    uint32_t tmem_base;
    int abort_flag;
};

__device__ __forceinline__ float gelu_erf(float x) {
    return x * 0.5f * (1.f + erff(x * 0.70710678118654752f));
}

template <int DT>
__device__ __forceinline__ void unpack16x2(uint32_t v, float& lo, float& hi) {
    if constexpr (DT == ADA_BF16) {
        lo = __uint_as_float(v << 16);
        hi = __uint_as_float(v & 0xFFFF0000u);
    } else {
        unpack_f16x2(v, lo, hi);
    }
}

template <int DT>
__device__ __forceinline__ uint32_t pack16x2(float lo, float hi) {
    if constexpr (DT == ADA_BF16) return pack_bf16x2(lo, hi);
    else return pack_f16x2(lo, hi);
}

// 64 columns of one output row, element by element, for outputs whose rows
// TMA cannot address (not 16-byte aligned); kept out of line.
template <int DT>
__device__ __noinline__ void epilogue_chunk_edge(const float* accv, const float* sbc, int act, const uint16_t* rrow,
                                                 uint16_t* yrow, int64_t col0, int64_t N) {
    for (int i = 0; i < 64 && col0 + i < N; ++i) {
        float v = round_to(accv[i] + sbc[i], DT);
        if (act == 1) v = round_to(gelu_erf(v), DT);
        if (rrow != nullptr) v = round_to(v + load_as_f32(rrow, col0 + i, DT), DT);
        store_from_f32(yrow, col0 + i, DT, v);
    }
}

template <int DT>
__global__ void __launch_bounds__(kLinThreads, 1) linear_tc_kernel(const __grid_constant__ LinearLaunch L) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sstg = base + kStages * kStageBytes;
    LinBarriers* bars = reinterpret_cast<LinBarriers*>(sstg + 8 * kStgBytes);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    const int n_m = static_cast<int>((L.M + kBM - 1) / kBM);
    const int n_n = static_cast<int>((L.N + kBN - 1) / kBN);
    const int64_t n_tiles = static_cast<int64_t>(n_m) * n_n;
    const int n_k = static_cast<int>((L.K + kBK - 1) / kBK);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(smem_u32(&bars->full[s]), 1);
            mbar_init(smem_u32(&bars->empty[s]), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(smem_u32(&bars->acc_full[a]), 1);
            mbar_init(smem_u32(&bars->acc_empty[a]), 256);
        }
        mbar_init(smem_u32(&bars->teardown), 1);
        for (int w = 0; w < 8; ++w) mbar_init(smem_u32(&bars->rfull[w]), 1);
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
    const uint32_t tmem = bars->tmem_base;
    volatile int* abort_flag = &bars->abort_flag;
    const uint64_t tmo = L.timeout_ns;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            tma_prefetch_desc(&L.tx);
            tma_prefetch_desc(&L.tw);
            uint32_t kc = 0;
            bool ok = true;
            for (int64_t t = blockIdx.x; ok && t < n_tiles; t += gridDim.x) {
                const int mt = static_cast<int>(t % n_m), nt = static_cast<int>(t / n_m);
                for (int kb = 0; kb < n_k; ++kb, ++kc) {
                    const uint32_t st = kc % kStages;
                    ok = mbar_wait(smem_u32(&bars->empty[st]), ((kc / kStages) & 1u) ^ 1u, abort_flag, tmo,
                                   L.status);
                    if (!ok) break;
                    const uint32_t fbar = smem_u32(&bars->full[st]);
                    mbar_arrive_expect_tx(fbar, kStageBytes);
                    uint8_t* sa = base + st * kStageBytes;
                    tma_load_2d(smem_u32(sa), &L.tx, fbar, kb * kBK, mt * kBM);
                    tma_load_2d(smem_u32(sa + kABytes), &L.tw, fbar, kb * kBK, nt * kBN);
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t fmt = DT == ADA_BF16 ? 1u : 0u;
            const uint32_t idesc = make_idesc(fmt, fmt, 0, 0, kBM, kBN);
            uint32_t kc = 0, tc = 0;
            bool ok = true;
            for (int64_t t = blockIdx.x; ok && t < n_tiles; t += gridDim.x, ++tc) {
                const uint32_t ab = tc & 1u;
                ok = mbar_wait(smem_u32(&bars->acc_empty[ab]), ((tc >> 1) & 1u) ^ 1u, abort_flag, tmo, L.status);
                if (!ok) break;
                tc_fence_after();
                const uint32_t acc = tmem + ab * kBN;
                for (int kb = 0; kb < n_k; ++kb, ++kc) {
                    const uint32_t st = kc % kStages;
                    ok = mbar_wait(smem_u32(&bars->full[st]), (kc / kStages) & 1u, abort_flag, tmo, L.status);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(base + st * kStageBytes);
                    const uint32_t b0 = a0 + kABytes;
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk)
                        mma_ss_f16(acc, make_sdesc_sw128(a0 + kk * 32, 16, 1024),
                                   make_sdesc_sw128(b0 + kk * 32, 16, 1024), idesc, (kb | kk) != 0 ? 1u : 0u);
                    tc_commit(smem_u32(&bars->empty[st]));
                }
                if (!ok) break;
                tc_commit(smem_u32(&bars->acc_full[ab]));
            }
            tc_commit(smem_u32(&bars->teardown));
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
    } else {
        // ---------------- epilogue ----------------
        // Per 64-column chunk each warp turns its 32 rows into a 32 x 64 tile
        // in its own shared-memory slot (128-byte swizzled rows, so the 16-byte
        // writes of 8 consecutive rows hit distinct banks) and one lane stores
        // it with TMA (rows past M, columns past N clipped). A residual tile
        // arrives in the same slot by TMA and is overwritten in place.
        const int quad = warp & 3;
        const int half = (warp - 2) >> 2;
        const int ew = warp - 2;
        const uint32_t lane_bits = static_cast<uint32_t>(quad * 32) << 16;
        const int act = L.act;
        const bool has_r = L.resid != nullptr;
        const bool tma_io = L.tma_io != 0;
        uint8_t* stg = sstg + ew * kStgBytes;
        const uint32_t stg_a = smem_u32(stg);
        const uint32_t rbar = smem_u32(&bars->rfull[ew]);
        uint32_t rph = 0;
        const int64_t N = L.N;
        uint32_t tc = 0;
        bool ok = true;
        for (int64_t t = blockIdx.x; ok && t < n_tiles; t += gridDim.x, ++tc) {
            const int mt = static_cast<int>(t % n_m), nt = static_cast<int>(t / n_m);
            const uint32_t ab = tc & 1u;
            // This warp's 128 bias values, lane l holding columns l, l+32, l+64,
            // l+96 (zero past N); broadcast by shuffles below.
            float breg[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int64_t col = static_cast<int64_t>(nt) * kBN + half * 128 + i * 32 + lane;
                breg[i] = (L.bias != nullptr && col < N) ? load_as_f32(L.bias, col, DT) : 0.f;
            }
            const int64_t row0 = static_cast<int64_t>(mt) * kBM + quad * 32;
            const uint32_t tacc = tmem + lane_bits + ab * kBN + half * 128;
            ok = mbar_wait(smem_u32(&bars->acc_full[ab]), (tc >> 1) & 1u, abort_flag, tmo, L.status);
            if (!ok) break;
            tc_fence_after();
#pragma unroll
            for (int c2 = 0; c2 < 2; ++c2) {
                const int64_t col0 = static_cast<int64_t>(nt) * kBN + half * 128 + c2 * 64;
                uint32_t r0[32], r1[32];
                tmem_ld32(tacc + c2 * 64, r0);
                tmem_ld32(tacc + c2 * 64 + 32, r1);
                if (tma_io) {
                    // While the accumulator loads are in flight: the slot is
                    // free once this warp's previous store has read it; then the
                    // residual tile may land in it.
                    if (lane == 0) {
                        bulk_wait_group_read0();
                        if (has_r) {
                            mbar_arrive_expect_tx(rbar, kStgBytes);
                            tma_load_2d(stg_a, &L.tr, rbar, static_cast<int>(col0), static_cast<int>(row0));
                        }
                    }
                    __syncwarp();
                }
                tmem_ld_wait();
                reg_fence32(r0);
                reg_fence32(r1);
                if (c2 == 1) {
                    // Both halves of this thread's columns are in registers:
                    // the accumulator buffer is free for the tile after next.
                    tc_fence_before();
                    mbar_arrive(smem_u32(&bars->acc_empty[ab]));
                }
                if (tma_io) {
                    // Linear (+ GELU) in registers, packed; then the residual.
                    uint32_t pk[32];
#pragma unroll
                    for (int g = 0; g < 8; ++g) {
                        float v[8];
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const float b = __shfl_sync(0xffffffffu, breg[c2 * 2 + g / 4], (g % 4) * 8 + i);
                            v[i] = round_to(__uint_as_float(g < 4 ? r0[g * 8 + i] : r1[(g - 4) * 8 + i]) + b, DT);
                        }
                        if (act == 1) {
#pragma unroll
                            for (int i = 0; i < 8; ++i) v[i] = round_to(gelu_erf(v[i]), DT);
                        }
#pragma unroll
                        for (int e = 0; e < 4; ++e) pk[g * 4 + e] = pack16x2<DT>(v[2 * e], v[2 * e + 1]);
                    }
                    if (has_r) {
                        ok = mbar_wait(rbar, rph, abort_flag, tmo, L.status);
                        rph ^= 1u;
                        if (!ok) break;
                    }
#pragma unroll
                    for (int g = 0; g < 8; ++g) {
                        uint4* cell = reinterpret_cast<uint4*>(stg + lane * 128 + ((g ^ (lane & 7)) * 16));
                        if (has_r) {
                            const uint4 rv = *cell;
                            const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                float x0, x1, y0, y1;
                                unpack16x2<DT>(rw[e], x0, x1);
                                unpack16x2<DT>(pk[g * 4 + e], y0, y1);
                                pk[g * 4 + e] = pack16x2<DT>(y0 + x0, y1 + x1);
                            }
                        }
                        *cell = make_uint4(pk[g * 4], pk[g * 4 + 1], pk[g * 4 + 2], pk[g * 4 + 3]);
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&L.ty, stg_a, static_cast<int>(col0), static_cast<int>(row0));
                        bulk_commit_group();
                    }
                } else {
                    float accv[64];
                    float bias64[64];
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        accv[i] = __uint_as_float(r0[i]);
                        accv[32 + i] = __uint_as_float(r1[i]);
                    }
#pragma unroll
                    for (int i = 0; i < 64; ++i)
                        bias64[i] = __shfl_sync(0xffffffffu, breg[c2 * 2 + i / 32], i % 32);
                    const int64_t grow = row0 + lane;
                    if (grow < L.M && col0 < N) {
                        const uint16_t* rrow =
                            has_r ? reinterpret_cast<const uint16_t*>(L.resid) + grow * L.ld_r : nullptr;
                        epilogue_chunk_edge<DT>(accv, bias64, act, rrow, reinterpret_cast<uint16_t*>(L.y) + grow * L.ld_y,
                                                col0, N);
                    }
                }
            }
        }
        // The last stores have read their tiles before the CTA leaves.
        if (lane == 0) bulk_wait_group0();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

}  // namespace

int launch_linear_tc(const LinearLaunch& L, cudaStream_t stream) {
    if (L.M <= 0 || L.N <= 0) return ADA_OK;
    if (L.dtype != ADA_BF16 && L.dtype != ADA_F16) return ADA_ERR_DTYPE;
    const bool bf = L.dtype == ADA_BF16;
    auto kern = bf ? linear_tc_kernel<ADA_BF16> : linear_tc_kernel<ADA_F16>;
    // Per process: the shared-memory opt-in of both instantiations, and the
    // SM count per device (launches stay cheap on the host).
    static const cudaError_t attr_bf =
        cudaFuncSetAttribute(linear_tc_kernel<ADA_BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, kLinSmem);
    static const cudaError_t attr_f16 =
        cudaFuncSetAttribute(linear_tc_kernel<ADA_F16>, cudaFuncAttributeMaxDynamicSharedMemorySize, kLinSmem);
    if ((bf ? attr_bf : attr_f16) != cudaSuccess) return ADA_ERR_LAUNCH;
    static int sm_count[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return ADA_ERR_LAUNCH;
    if (sm_count[dev] <= 0) {
        int sms = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
            return ADA_ERR_LAUNCH;
        sm_count[dev] = sms;
    }
    const int64_t tiles = ((L.M + kBM - 1) / kBM) * ((L.N + kBN - 1) / kBN);
    const int64_t grid = tiles < sm_count[dev] ? tiles : sm_count[dev];
    kern<<<static_cast<unsigned>(grid), kLinThreads, kLinSmem, stream>>>(L);
    return cudaGetLastError() == cudaSuccess ? ADA_OK : ADA_ERR_LAUNCH;
}

}  // namespace ada
