// The dense layers on either side of the attention path on the sm_100a tensor
// cores: y = act(x W^T + b) (+ r), the nn.Linear of the module's q/k/v
// projection and out_proj (src/adaattn/attention/adaattn.py:411-418 and :457)
// and of the transformer block that hosts it (its feed-forward and residual
// sums, examples/transformer_integration.py:33-58).
//
// x [M, K] and W [N, K] are 16-bit (both the same type), rows K-contiguous, so
// both operands are K-major. CTA pairs (clusters of two, one CTA per SM,
// persistent) walk 256 x 256 output tiles, N-fastest when x is the larger
// operand (the pairs running together share one 256-row block of x, which
// is read from HBM once; W stays in L2), else M-fastest. Each tile is one
// chain of cta_group::2 tcgen05 MMAs (M = 256, N = 256, K = 16): CTA r of the
// pair loads rows 128 r .. +127 of the tile's x block and rows 128 r .. +127
// of its W block, 64-column K blocks through a 5-stage shared-memory ring
// filled by TMA, so each SM streams half of the W tile (the pair splits the
// shared-memory operand traffic of a 128 x 256 single-CTA tile in half). The
// even CTA's MMA thread issues the products once both halves of a stage have
// landed (both CTAs' TMA loads count their bytes on its barrier); each CTA
// keeps its 128 rows of the fp32 accumulator in its own tensor memory,
// double buffered (2 x 256 columns = all 512), so a tile's epilogue overlaps
// the next tile's products.
//
// Epilogue, per element, in the order the reference's PyTorch ops round:
//   t = round(acc + b)                   nn.Linear's output in the inputs' dtype
//   t = round(gelu(t))                   nn.GELU (erf form), when asked
//   t = round(t + r)                     the residual sum, when asked
// Warp roles (576 threads per CTA): warp 0 TMA producer, warp 1 TMEM
// allocation and (even CTA) MMA issue, warps 2-17 epilogue in two groups of
// eight, group g draining the tiles of accumulator buffer g (every other
// tile), so two tiles' epilogues run at once and hide each other's latency
// (a GELU epilogue is as long as a K = 768 main loop). Warp w reads TMEM lanes
// 32 (w mod 4) .. +31, one output row per thread, and columns
// 128 (((w - 2) mod 8) / 4) .. +127 of its tile. Every wait is bounded
// (ada::mbar_wait): a timeout raises the CTA's abort flag and ADA_ERR_TIMEOUT
// in the status word.
#include "ada_common.cuh"
#include "ada_internal.h"

namespace ada {
namespace {

constexpr int kLinThreads = 576;  // warps 0-1 TMA and MMA, warps 2-17 two epilogue groups
constexpr int kBM = 128;                      // rows of the tile per CTA (256 per pair)
constexpr int kPairM = 256;
constexpr int kBN = 256;                      // columns of the tile
constexpr int kBNh = 128;                     // rows of W per CTA
constexpr int kBK = 64;                       // 16-bit elements per 128-byte swizzle atom
constexpr int kStages = 5;
constexpr int kABytes = kBM * kBK * 2;        // 16 KB
constexpr int kBBytes = kBNh * kBK * 2;       // 16 KB
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kStgBytes = 32 * 128;          // one 32-row x 64-column output tile
constexpr int kLinSmem = kStages * kStageBytes + 16 * kStgBytes + 1024 + 256;  // one tile per epilogue warp

struct __align__(8) LinBarriers {
    uint64_t full[kStages];
    uint64_t empty[kStages];
    uint64_t acc_full[2];
    uint64_t acc_empty[2];
    uint64_t teardown;
    uint64_t rfull[16];  // per epilogue warp: its residual tile has landed
    // full[] and acc_empty[] are used on the even CTA only (the odd CTA's TMA
    // loads and epilogue warps count on the even CTA's copies).
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

// Output tile t -> (M tile, N tile): the N tiles of one x row block side by
// side (n_fastest), or the M tiles of one W column block side by side. The
// pairs running together then share one operand block through L2, and the
// operand that is larger in HBM is the one read from it once.
__device__ __forceinline__ int tile_m(int64_t t, int n_m, int n_n, bool n_fastest) {
    return static_cast<int>(n_fastest ? t / n_n : t % n_m);
}
__device__ __forceinline__ int tile_n(int64_t t, int n_m, int n_n, bool n_fastest) {
    return static_cast<int>(n_fastest ? t % n_n : t / n_m);
}

// The barrier at this shared-memory offset in both CTAs of the pair receives
// one arrival when the issuing thread's products so far have completed.
__device__ __forceinline__ void commit_both(uint32_t bar) {
    tc_commit_pair(mapa_shared(bar, 0));
    tc_commit_pair(mapa_shared(bar, 1));
}

template <int DT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kLinThreads, 1)
    linear_tc_kernel(const __grid_constant__ LinearLaunch L) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sstg = base + kStages * kStageBytes;
    LinBarriers* bars = reinterpret_cast<LinBarriers*>(sstg + 16 * kStgBytes);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int pair = static_cast<int>(blockIdx.x >> 1), n_pairs = static_cast<int>(gridDim.x >> 1);

    const int n_m = static_cast<int>((L.M + kPairM - 1) / kPairM);
    const int n_n = static_cast<int>((L.N + kBN - 1) / kBN);
    const int64_t n_tiles = static_cast<int64_t>(n_m) * n_n;
    const int n_k = static_cast<int>((L.K + kBK - 1) / kBK);
    const bool nfast = L.n_fastest != 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(smem_u32(&bars->full[s]), 1);
            mbar_init(smem_u32(&bars->empty[s]), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(smem_u32(&bars->acc_full[a]), 1);
            mbar_init(smem_u32(&bars->acc_empty[a]), 16);  // one arrival per epilogue warp of the pair
        }
        mbar_init(smem_u32(&bars->teardown), 1);
        for (int w = 0; w < 16; ++w) mbar_init(smem_u32(&bars->rfull[w]), 1);
        bars->abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_u32(&bars->tmem_base), 512);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    // Both CTAs' barriers are initialised before either signals the other's.
    cluster_sync_all();
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
            for (int64_t t = pair; ok && t < n_tiles; t += n_pairs) {
                const int mt = tile_m(t, n_m, n_n, nfast), nt = tile_n(t, n_m, n_n, nfast);
                const int xrow = mt * kPairM + static_cast<int>(rank) * kBM;
                const int wrow = nt * kBN + static_cast<int>(rank) * kBNh;
                for (int kb = 0; kb < n_k; ++kb, ++kc) {
                    const uint32_t st = kc % kStages;
                    ok = mbar_wait(smem_u32(&bars->empty[st]), ((kc / kStages) & 1u) ^ 1u, abort_flag, tmo,
                                   L.status);
                    if (!ok) break;
                    // Both CTAs' bytes complete on the even CTA's barrier.
                    const uint32_t fbar_local = smem_u32(&bars->full[st]);
                    if (rank == 0) mbar_arrive_expect_tx(fbar_local, 2 * kStageBytes);
                    const uint32_t fbar = mapa_shared(fbar_local, 0);
                    uint8_t* sa = base + st * kStageBytes;
                    tma_load_2d_pair(smem_u32(sa), &L.tx, fbar, kb * kBK, xrow);
                    tma_load_2d_pair(smem_u32(sa + kABytes), &L.tw, fbar, kb * kBK, wrow);
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0 && rank == 0) {
            constexpr uint32_t fmt = DT == ADA_BF16 ? 1u : 0u;
            const uint32_t idesc = make_idesc(fmt, fmt, 0, 0, kPairM, kBN);
            uint32_t kc = 0, tc = 0;
            bool ok = true;
            for (int64_t t = pair; ok && t < n_tiles; t += n_pairs, ++tc) {
                const uint32_t ab = tc & 1u;
                // Both CTAs' epilogues have read this accumulator buffer.
                ok = mbar_wait_cluster(smem_u32(&bars->acc_empty[ab]), ((tc >> 1) & 1u) ^ 1u, abort_flag, tmo,
                                       L.status);
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
                        mma_ss_f16_pair(acc, make_sdesc_sw128(a0 + kk * 32, 16, 1024),
                                        make_sdesc_sw128(b0 + kk * 32, 16, 1024), idesc, (kb | kk) != 0 ? 1u : 0u);
                    commit_both(smem_u32(&bars->empty[st]));
                }
                if (!ok) break;
                commit_both(smem_u32(&bars->acc_full[ab]));
            }
            commit_both(smem_u32(&bars->teardown));
        }
        if (lane == 0) {
            // Both CTAs: every product of the pair has completed (they write
            // this CTA's tensor memory and read its shared memory).
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
        const int ew = warp - 2;
        const int grp = ew >> 3;          // accumulator buffer this warp drains
        const int half = (ew & 7) >> 2;
        const uint32_t lane_bits = static_cast<uint32_t>(quad * 32) << 16;
        const int act = L.act;
        const bool has_r = L.resid != nullptr;
        const bool tma_io = L.tma_io != 0;
        uint8_t* stg_w = sstg + ew * kStgBytes;  // this warp's slot
        const uint32_t rbar = smem_u32(&bars->rfull[ew]);
        uint32_t rph = 0;
        const int64_t N = L.N;
        uint32_t tc = 0;
        bool ok = true;
        // The even CTA's acc_empty barriers, where this warp reports a drained buffer.
        const uint32_t acc_empty0 = mapa_shared(smem_u32(&bars->acc_empty[0]), 0);
        for (int64_t t = pair; ok && t < n_tiles; t += n_pairs, ++tc) {
            const uint32_t ab = tc & 1u;
            if (static_cast<int>(ab) != grp) continue;  // the other group's tile
            const int mt = tile_m(t, n_m, n_n, nfast), nt = tile_n(t, n_m, n_n, nfast);
            // This warp's 128 bias values, lane l holding columns l, l+32, l+64,
            // l+96 (zero past N); broadcast by shuffles below.
            float breg[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int64_t col = static_cast<int64_t>(nt) * kBN + half * 128 + i * 32 + lane;
                breg[i] = (L.bias != nullptr && col < N) ? load_as_f32(L.bias, col, DT) : 0.f;
            }
            const int64_t row0 = static_cast<int64_t>(mt) * kPairM + rank * kBM + quad * 32;
            const uint32_t tacc = tmem + lane_bits + ab * kBN + half * 128;
            ok = mbar_wait(smem_u32(&bars->acc_full[ab]), (tc >> 1) & 1u, abort_flag, tmo, L.status);
            if (!ok) break;
            tc_fence_after();
#pragma unroll
            for (int c2 = 0; c2 < 2; ++c2) {
                const int64_t col0 = static_cast<int64_t>(nt) * kBN + half * 128 + c2 * 64;
                // A tile that lies wholly past M or N (the odd CTA's rows of a
                // last, partial pair tile) is neither loaded nor stored.
                const bool live = row0 < L.M && col0 < N;
                // One slot per warp: the previous chunk's store must have read
                // it before this chunk (or its residual tile) is written.
                uint8_t* stg = stg_w;
                const uint32_t stg_a = smem_u32(stg);
                uint32_t r0[32], r1[32];
                tmem_ld32(tacc + c2 * 64, r0);
                tmem_ld32(tacc + c2 * 64 + 32, r1);
                if (tma_io) {
                    // While the accumulator loads are in flight: the slot is
                    // free once this warp's previous store has read it; then the
                    // residual tile may land in it.
                    if (lane == 0) {
                        bulk_wait_group_read0();
                        if (has_r && live) {
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
                    // Both halves of this warp's columns are in registers: the
                    // accumulator buffer is free for the tile after next.
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cluster(acc_empty0 + ab * 8);
                }
                if (tma_io) {
                    // Linear (+ GELU) in registers, packed; then the residual.
                    // Without GELU the Linear's rounding is the packing itself.
                    uint32_t pk[32];
                    if (act == 1) {
#pragma unroll
                        for (int g = 0; g < 8; ++g) {
                            float v[8];
#pragma unroll
                            for (int i = 0; i < 8; ++i) {
                                const float b = __shfl_sync(0xffffffffu, breg[c2 * 2 + g / 4], (g % 4) * 8 + i);
                                v[i] = round_to(gelu_erf(round_to(
                                                    __uint_as_float(g < 4 ? r0[g * 8 + i] : r1[(g - 4) * 8 + i]) + b, DT)),
                                                DT);
                            }
#pragma unroll
                            for (int e = 0; e < 4; ++e) pk[g * 4 + e] = pack16x2<DT>(v[2 * e], v[2 * e + 1]);
                        }
                    } else {
#pragma unroll
                        for (int e = 0; e < 32; ++e) {
                            const int c = 2 * e;  // column pair within the chunk
                            const float b0 = __shfl_sync(0xffffffffu, breg[c2 * 2 + c / 32], c % 32);
                            const float b1 = __shfl_sync(0xffffffffu, breg[c2 * 2 + c / 32], c % 32 + 1);
                            const uint32_t a0 = c < 32 ? r0[c] : r1[c - 32];
                            const uint32_t a1 = c < 32 ? r0[c + 1] : r1[c - 31];
                            float y0, y1;
                            f2_unpack(f2_add(f2_pack(__uint_as_float(a0), __uint_as_float(a1)), f2_pack(b0, b1)), y0, y1);
                            pk[e] = pack16x2<DT>(y0, y1);
                        }
                    }
                    if (has_r && live) {
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
                        // One bulk group per chunk (empty when nothing is
                        // stored) keeps the slot accounting above exact.
                        if (live) tma_store_2d(&L.ty, stg_a, static_cast<int>(col0), static_cast<int>(row0));
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
        tmem_dealloc_pair(tmem, 512);
    }
    // Neither CTA leaves while the other may still signal its barriers.
    cluster_sync_all();
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
    const int64_t tiles = ((L.M + kPairM - 1) / kPairM) * ((L.N + kBN - 1) / kBN);
    const int64_t pairs = sm_count[dev] / 2;
    const int64_t grid = 2 * (tiles < pairs ? tiles : pairs);
    kern<<<static_cast<unsigned>(grid), kLinThreads, kLinSmem, stream>>>(L);
    return cudaGetLastError() == cudaSuccess ? ADA_OK : ADA_ERR_LAUNCH;
}

}  // namespace ada
