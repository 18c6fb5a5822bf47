// K2: fused attention forward on the sm_100a tensor cores.
//
// One CTA owns two 128-row query tiles of one (b, h) and streams 128-key
// blocks of K and V through a shared-memory ring filled by TMA. S = Q K^T and
// O += P V run as tcgen05 MMAs with fp32 accumulators in tensor memory; the
// score block never leaves the SM. Warp roles (320 threads):
//   warps 0-3 / 4-7  softmax for query tile 0 / 1: read S from TMEM (one row
//                    per thread), online softmax in registers, write P (16-bit
//                    or E4M3) back into the S columns, rescale O when the
//                    running maximum moves, final normalisation and store.
//   warp 8           TMA producer (Q tiles once, then K_j, V_j per block).
//   warp 9           TMEM allocation and the single-thread MMA issuer.
// The two query tiles ping-pong: while one tile's softmax runs, the tensor
// core works on the other tile's products.
//
// TMEM columns: S0 [0,128) S1 [128,256) O0 [256,256+DV) O1 [256+DV,256+2DV).
// Every wait is bounded (ada::mbar_wait); a timeout raises the CTA's abort
// flag and ADA_ERR_TIMEOUT in the status word instead of hanging.
#include "ada_common.cuh"
#include "ada_internal.h"

namespace ada {
namespace {

constexpr int kThreadsTc = 320;
constexpr int kSmemTarget = 200 * 1024;

template <int ELT, int DQK, int DV>
struct TcCfg {
    static constexpr int EB = (ELT == 2) ? 1 : 2;
    static constexpr int BM = 128;
    static constexpr int BN = 128;
    static constexpr int BOX = 128 * 128;  // bytes of one 128-row x 128-byte TMA box
    static constexpr int ATOM_COLS = 128 / EB;
    static constexpr int QK_ATOMS = DQK * EB / 128;
    static constexpr int V_ATOMS = DV * EB / 128;
    static_assert(QK_ATOMS >= 1 && QK_ATOMS * 128 == DQK * EB, "DQK row must be whole 128-byte atoms");
    static_assert(V_ATOMS >= 1 && V_ATOMS * 128 == DV * EB, "DV row must be whole 128-byte atoms");
    static constexpr int Q_BYTES = BM * DQK * EB;
    static constexpr int K_BYTES = BN * DQK * EB;
    static constexpr int V_BYTES = BN * DV * EB;
    static constexpr int STAGE_BYTES = K_BYTES > V_BYTES ? K_BYTES : V_BYTES;
    static constexpr int NSTAGE_RAW = (kSmemTarget - 2 * Q_BYTES) / STAGE_BYTES;
    static constexpr int NSTAGE = NSTAGE_RAW > 8 ? 8 : NSTAGE_RAW;
    static_assert(NSTAGE >= 2, "ring too small");
    static constexpr int MMA_K = (ELT == 2) ? 32 : 16;   // elements per MMA k-step
    static constexpr int KSTEP_BYTES = MMA_K * EB;        // 32 bytes either way
    static constexpr int P_COLS = BN * EB / 4;            // TMEM columns holding P
    static constexpr uint32_t FMT = (ELT == 1) ? 1u : 0u; // bf16 = 1, f16 = 0, e4m3 = 0
    static constexpr uint32_t IDESC_QK = make_idesc(FMT, FMT, 0, 0, 128, BN);
    static constexpr uint32_t IDESC_PV = make_idesc(FMT, FMT, 0, 1, 128, DV);
    static constexpr int SMEM_BYTES = 2 * Q_BYTES + NSTAGE * STAGE_BYTES + 1024 /*align*/ + 256;
};

struct __align__(8) TcBarriers {
    uint64_t q_full;
    uint64_t s_full[2];
    uint64_t p_full[2];
    uint64_t o_full[2];
    uint64_t teardown;
    uint64_t kv_full[8];
    uint64_t kv_empty[8];
    uint32_t tmem_base;
    int abort_flag;
};

__device__ __forceinline__ int ceil_div_i(int64_t a, int64_t b) { return static_cast<int>((a + b - 1) / b); }

template <int ELT>
__device__ __forceinline__ void issue_mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                             uint32_t acc) {
    if constexpr (ELT == 2)
        mma_ss_f8(d, a, b, idesc, acc);
    else
        mma_ss_f16(d, a, b, idesc, acc);
}
template <int ELT>
__device__ __forceinline__ void issue_mma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc,
                                             uint32_t acc) {
    if constexpr (ELT == 2)
        mma_ts_f8(d, a, b, idesc, acc);
    else
        mma_ts_f16(d, a, b, idesc, acc);
}

// Wait that ignores the abort flag but is still bounded; used on the way out
// so the CTA never frees tensor memory under an MMA that is still running.
__device__ __forceinline__ void teardown_wait(uint32_t bar, uint32_t parity, uint64_t timeout_ns,
                                              unsigned int* status) {
    const uint64_t t0 = globaltimer_ns();
    uint32_t spins = 0;
    while (!mbar_try_wait(bar, parity)) {
        if ((++spins & 63u) == 0u && globaltimer_ns() - t0 > timeout_ns) {
            record_error(status, ADA_ERR_TIMEOUT);
            return;
        }
    }
}

template <int ELT, int DQK, int DV>
__global__ void __launch_bounds__(kThreadsTc, 1) fmha_tc_kernel(const __grid_constant__ TcLaunch L) {
    using C = TcCfg<ELT, DQK, DV>;
    extern __shared__ uint8_t smem_raw[];

    const int64_t BH = L.B * L.H;
    const int n_qt = ceil_div_i(L.Nq, 128);
    const int n_qtp = (n_qt + 1) / 2;
    const int64_t lin = blockIdx.x;
    const int64_t bh = lin % BH;
    const int qtp = n_qtp - 1 - static_cast<int>(lin / BH);  // heavy (late) tiles first
    if (!head_selected(L.sel, bh)) return;                    // whole CTA, before any sync
    const int b = static_cast<int>(bh / L.H);
    const int h = static_cast<int>(bh % L.H);

    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = base;
    uint8_t* sKV = base + 2 * C::Q_BYTES;
    TcBarriers* bars = reinterpret_cast<TcBarriers*>(sKV + C::NSTAGE * C::STAGE_BYTES);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    // Key blocks each query tile needs.
    const int nkb = ceil_div_i(L.Nk, 128);
    int n_t[2];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
        const int64_t r0 = (static_cast<int64_t>(qtp) * 2 + t) * 128;
        if (r0 >= L.Nq) {
            n_t[t] = 0;
        } else if (L.causal) {
            const int64_t r_last = (r0 + 127 < L.Nq - 1) ? r0 + 127 : L.Nq - 1;
            const int need = static_cast<int>(r_last / 128) + 1;
            n_t[t] = need < nkb ? need : nkb;
        } else {
            n_t[t] = nkb;
        }
    }
    const int nblk = n_t[0] > n_t[1] ? n_t[0] : n_t[1];

    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&bars->q_full), 1);
        for (int t = 0; t < 2; ++t) {
            mbar_init(smem_u32(&bars->s_full[t]), 1);
            mbar_init(smem_u32(&bars->p_full[t]), 128);
            mbar_init(smem_u32(&bars->o_full[t]), 1);
        }
        mbar_init(smem_u32(&bars->teardown), 1);
        for (int s = 0; s < C::NSTAGE; ++s) {
            mbar_init(smem_u32(&bars->kv_full[s]), 1);
            mbar_init(smem_u32(&bars->kv_empty[s]), 1);
        }
        bars->abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 9) {
        tmem_alloc(smem_u32(&bars->tmem_base), 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;
    volatile int* abort_flag = &bars->abort_flag;
    const uint64_t tmo = L.timeout_ns;

    if (warp == 8) {
        // ---------------- TMA producer ----------------
        if (lane == 0 && nblk > 0) {
            tma_prefetch_desc(&L.tq);
            tma_prefetch_desc(&L.tk);
            tma_prefetch_desc(&L.tv);
            const uint32_t qbar = smem_u32(&bars->q_full);
            mbar_arrive_expect_tx(qbar, 2 * C::Q_BYTES);
            for (int t = 0; t < 2; ++t)
                for (int a = 0; a < C::QK_ATOMS; ++a)
                    tma_load_4d(smem_u32(sQ + t * C::Q_BYTES + a * C::BOX), &L.tq, qbar,
                                a * C::ATOM_COLS, (qtp * 2 + t) * 128, h, b);
            for (int j = 0; j < nblk; ++j) {
                for (int half = 0; half < 2; ++half) {
                    const int idx = 2 * j + half;
                    const int st = idx % C::NSTAGE;
                    const uint32_t ph = (idx / C::NSTAGE) & 1;
                    if (!mbar_wait(smem_u32(&bars->kv_empty[st]), ph ^ 1u, abort_flag, tmo, L.status))
                        break;
                    const uint32_t fbar = smem_u32(&bars->kv_full[st]);
                    uint8_t* dst = sKV + st * C::STAGE_BYTES;
                    if (half == 0) {
                        mbar_arrive_expect_tx(fbar, C::K_BYTES);
                        for (int a = 0; a < C::QK_ATOMS; ++a)
                            tma_load_4d(smem_u32(dst + a * C::BOX), &L.tk, fbar, a * C::ATOM_COLS,
                                        j * 128, h, b);
                    } else {
                        mbar_arrive_expect_tx(fbar, C::V_BYTES);
                        for (int a = 0; a < C::V_ATOMS; ++a)
                            tma_load_4d(smem_u32(dst + a * C::BOX), &L.tv, fbar, a * C::ATOM_COLS,
                                        j * 128, h, b);
                    }
                }
                if (*abort_flag) break;
            }
        }
        __syncwarp();
    } else if (warp == 9) {
        // ---------------- MMA issuer ----------------
        if (lane == 0 && nblk > 0) {
            const uint32_t sQa = smem_u32(sQ);
            const uint32_t sKVa = smem_u32(sKV);
            bool ok = mbar_wait(smem_u32(&bars->q_full), 0, abort_flag, tmo, L.status);
            auto issue_s = [&](int t, int stage) {
                const uint32_t q0 = sQa + t * C::Q_BYTES;
                const uint32_t k0 = sKVa + stage * C::STAGE_BYTES;
#pragma unroll
                for (int ks = 0; ks < DQK / C::MMA_K; ++ks) {
                    const int byte = ks * C::KSTEP_BYTES;
                    const uint32_t off = (byte / 128) * C::BOX + (byte % 128);
                    const uint64_t ad = make_sdesc_sw128(q0 + off, 16, 1024);
                    const uint64_t bd = make_sdesc_sw128(k0 + off, 16, 1024);
                    issue_mma_ss<ELT>(tmem + t * 128, ad, bd, C::IDESC_QK, ks > 0 ? 1u : 0u);
                }
                tc_commit(smem_u32(&bars->s_full[t]));
            };
            auto issue_pv = [&](int t, int stage, bool first) {
                const uint32_t v0 = sKVa + stage * C::STAGE_BYTES;
#pragma unroll
                for (int ks = 0; ks < C::BN / C::MMA_K; ++ks) {
                    const uint64_t bd = make_sdesc_sw128(v0 + ks * C::MMA_K * 128, C::BOX, 1024);
                    const uint32_t a_t = tmem + t * 128 + ks * (C::MMA_K * C::EB / 4);
                    issue_mma_ts<ELT>(tmem + 256 + t * DV, a_t, bd, C::IDESC_PV,
                                      (!first || ks > 0) ? 1u : 0u);
                }
            };
            if (ok) {
                // K_0 and the first score blocks.
                ok = mbar_wait(smem_u32(&bars->kv_full[0]), 0, abort_flag, tmo, L.status);
                if (ok) {
                    tc_fence_after();
                    for (int t = 0; t < 2; ++t)
                        if (n_t[t] > 0) issue_s(t, 0);
                    tc_commit(smem_u32(&bars->kv_empty[0]));
                }
            }
            for (int j = 0; ok && j < nblk; ++j) {
                const int iv = 2 * j + 1;
                const int sv = iv % C::NSTAGE;
                ok = mbar_wait(smem_u32(&bars->kv_full[sv]), (iv / C::NSTAGE) & 1, abort_flag, tmo,
                               L.status);
                if (!ok) break;
                tc_fence_after();
                const int ik = 2 * j + 2;
                const int sk = ik % C::NSTAGE;
                bool k_ready = false;
                for (int t = 0; t < 2 && ok; ++t) {
                    if (j < n_t[t]) {
                        ok = mbar_wait(smem_u32(&bars->p_full[t]), j & 1, abort_flag, tmo, L.status);
                        if (!ok) break;
                        tc_fence_after();
                        issue_pv(t, sv, j == 0);
                        if (j == n_t[t] - 1) tc_commit(smem_u32(&bars->o_full[t]));
                    }
                    if (j + 1 < n_t[t]) {
                        if (!k_ready) {
                            ok = mbar_wait(smem_u32(&bars->kv_full[sk]), (ik / C::NSTAGE) & 1,
                                           abort_flag, tmo, L.status);
                            if (!ok) break;
                            tc_fence_after();
                            k_ready = true;
                        }
                        issue_s(t, sk);
                    }
                }
                tc_commit(smem_u32(&bars->kv_empty[sv]));
                if (k_ready) tc_commit(smem_u32(&bars->kv_empty[sk]));
            }
            // Everything issued so far completes before the CTA frees TMEM.
            tc_commit(smem_u32(&bars->teardown));
            teardown_wait(smem_u32(&bars->teardown), 0, tmo, L.status);
        }
        __syncwarp();
    } else {
        // ---------------- softmax warpgroups ----------------
        const int t = warp >> 2;
        const int row = (warp & 3) * 32 + lane;  // TMEM lane == row of the tile
        const int64_t qrow = (static_cast<int64_t>(qtp) * 2 + t) * 128 + row;
        const uint32_t lane_bits = static_cast<uint32_t>((warp & 3) * 32) << 16;
        const uint32_t tS = tmem + lane_bits + t * 128;
        const uint32_t tO = tmem + lane_bits + 256 + t * DV;
        const int nt = n_t[t];
        const int64_t tile_r0 = (static_cast<int64_t>(qtp) * 2 + t) * 128;
        float sq = 1.f;
        if constexpr (ELT == 2) {
            if (nt > 0) sq = L.q_scale[bh * L.nt_q + (qtp * 2 + t)];  // tile exists
        }
        float m_run = -INFINITY;
        float l_run = 0.f;
        bool ok = true;
        for (int j = 0; j < nt; ++j) {
            ok = mbar_wait(smem_u32(&bars->s_full[t]), j & 1, abort_flag, tmo, L.status);
            if (!ok) break;
            tc_fence_after();
            float s[128];
            {
                uint32_t r[32];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    tmem_ld32(tS + c * 32, r);
                    tmem_ld_wait();
                    reg_fence32(r);
#pragma unroll
                    for (int i = 0; i < 32; ++i) s[c * 32 + i] = __uint_as_float(r[i]);
                }
            }
            float sl2 = L.scale_log2;
            if constexpr (ELT == 2) sl2 *= sq * L.k_scale[bh * L.nt_k + j];
            const int64_t kv0 = static_cast<int64_t>(j) * 128;
            const bool edge = (kv0 + 128 > L.Nk) || (L.causal && kv0 + 127 > tile_r0);
            if (edge) {
#pragma unroll
                for (int c = 0; c < 128; ++c) {
                    const int64_t kv = kv0 + c;
                    if (kv >= L.Nk || (L.causal && kv > qrow)) s[c] = -INFINITY;
                }
            }
            if (L.mask.data != nullptr && qrow < L.Nq) {
                // logits are s * scale + m; in raw-score units that is s + m / scale.
                const float inv_scale = 1.f / (sl2 * 0.69314718056f);
                const int64_t mb = b * L.mask.s[0] + h * L.mask.s[1] + qrow * L.mask.s[2];
#pragma unroll
                for (int c = 0; c < 128; ++c) {
                    const int64_t kv = kv0 + c;
                    if (kv < L.Nk) {
                        const float mv = load_as_f32(L.mask.data, mb + kv * L.mask.s[3], L.mask.dtype);
                        if (L.mask.dtype == ADA_BOOL) {
                            if (mv == 0.f) s[c] = -INFINITY;
                        } else {
                            s[c] += round_to(mv, L.round_dtype) * inv_scale;
                        }
                    }
                }
            }
            float mx[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) mx[i] = s[i];
#pragma unroll
            for (int c = 8; c < 128; ++c) mx[c & 7] = fmaxf(mx[c & 7], s[c]);
            const float m_blk = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                                      fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
            const float m_cand = m_blk * sl2;
            float m_new = m_run;
            if constexpr (ELT == 2) {
                m_new = fmaxf(m_run, m_cand);
            } else {
                // Keep a stale maximum until it falls 8 (log2 units) behind:
                // P stays <= 256, exact in 16-bit, and O is rescaled rarely.
                if (m_cand > m_run + 8.f) m_new = m_cand;
            }
            const float alpha = (m_new == m_run) ? 1.f : fast_exp2(m_run - m_new);
            const float neg_m = (m_new == -INFINITY) ? 0.f : -m_new;
            float ls[4] = {0.f, 0.f, 0.f, 0.f};
            {
                constexpr int NP = C::P_COLS / 32;  // 32-column chunks of P
                uint32_t pr[32];
#pragma unroll
                for (int chunk = 0; chunk < NP; ++chunk) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        if constexpr (ELT == 2) {
                            const int c = chunk * 128 + i * 4;
                            float p0 = fast_exp2(fmaf(s[c + 0], sl2, neg_m));
                            float p1 = fast_exp2(fmaf(s[c + 1], sl2, neg_m));
                            float p2 = fast_exp2(fmaf(s[c + 2], sl2, neg_m));
                            float p3 = fast_exp2(fmaf(s[c + 3], sl2, neg_m));
                            ls[0] += p0;
                            ls[1] += p1;
                            ls[2] += p2;
                            ls[3] += p3;
                            pr[i] = pack_e4m3x4(p0 * 448.f, p1 * 448.f, p2 * 448.f, p3 * 448.f);
                        } else {
                            const int c = chunk * 64 + i * 2;
                            float p0 = fast_exp2(fmaf(s[c + 0], sl2, neg_m));
                            float p1 = fast_exp2(fmaf(s[c + 1], sl2, neg_m));
                            ls[i & 1] += p0;
                            ls[2 + (i & 1)] += p1;
                            pr[i] = (ELT == 1) ? pack_bf16x2(p0, p1) : pack_f16x2(p0, p1);
                        }
                    }
                    tmem_st32(tS + chunk * 32, pr);
                }
            }
            l_run = l_run * alpha + ((ls[0] + ls[1]) + (ls[2] + ls[3]));
            if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
                uint32_t r[32];
#pragma unroll
                for (int c = 0; c < DV / 32; ++c) {
                    tmem_ld32(tO + c * 32, r);
                    tmem_ld_wait();
                    reg_fence32(r);
#pragma unroll
                    for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
                    tmem_st32(tO + c * 32, r);
                }
            }
            m_run = m_new;
            tmem_st_wait();
            tc_fence_before();
            mbar_arrive(smem_u32(&bars->p_full[t]));
        }
        if (nt > 0 && ok) {
            ok = mbar_wait(smem_u32(&bars->o_full[t]), 0, abort_flag, tmo, L.status);
        }
        if (nt > 0 && ok) {
            tc_fence_after();
            float post = 1.f / l_run;
            if constexpr (ELT == 2) post *= L.v_scale[bh] * (1.f / 448.f);
            const bool row_ok = qrow < L.Nq;
            uint8_t* orow = reinterpret_cast<uint8_t*>(L.out);
            const int64_t obase = b * L.os[0] + h * L.os[1] + qrow * L.os[2];
            uint32_t r[32];
#pragma unroll
            for (int c = 0; c < DV / 32; ++c) {
                tmem_ld32(tO + c * 32, r);
                tmem_ld_wait();
                reg_fence32(r);
                if (row_ok) {
                    float o[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] = round_to(__uint_as_float(r[i]) * post, L.round_dtype);
                    const int col0 = c * 32;
                    if (L.out_vec && col0 + 32 <= L.dv_out) {
                        if (L.out_dtype == ADA_F32) {
                            float4* dst = reinterpret_cast<float4*>(orow + (obase + col0) * 4);
#pragma unroll
                            for (int i = 0; i < 8; ++i)
                                dst[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
                        } else {
                            uint4* dst = reinterpret_cast<uint4*>(orow + (obase + col0) * 2);
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                uint32_t w[4];
#pragma unroll
                                for (int k2 = 0; k2 < 4; ++k2) {
                                    const float lo = o[8 * i + 2 * k2], hi = o[8 * i + 2 * k2 + 1];
                                    w[k2] = (L.out_dtype == ADA_BF16) ? pack_bf16x2(lo, hi) : pack_f16x2(lo, hi);
                                }
                                dst[i] = make_uint4(w[0], w[1], w[2], w[3]);
                            }
                        }
                    } else {
                        for (int i = 0; i < 32; ++i)
                            if (col0 + i < L.dv_out)
                                store_from_f32(L.out, obase + (col0 + i) * L.os[3], L.out_dtype, o[i]);
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 9) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

template <int ELT, int DQK, int DV>
int launch_variant(const TcLaunch& L, cudaStream_t stream) {
    using C = TcCfg<ELT, DQK, DV>;
    auto kern = fmha_tc_kernel<ELT, DQK, DV>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES) !=
        cudaSuccess)
        return ADA_ERR_LAUNCH;
    const int64_t n_qt = (L.Nq + 127) / 128;
    const int64_t n_qtp = (n_qt + 1) / 2;
    const int64_t grid = n_qtp * L.B * L.H;
    if (grid <= 0) return ADA_OK;
    if (grid > 0x7fffffffLL) return ADA_ERR_UNSUPPORTED;
    kern<<<static_cast<unsigned>(grid), kThreadsTc, C::SMEM_BYTES, stream>>>(L);
    return cudaGetLastError() == cudaSuccess ? ADA_OK : ADA_ERR_LAUNCH;
}

}  // namespace

int launch_fmha_tc(const TcLaunch& L, cudaStream_t stream) {
    if (L.elt == 2) {
        if (L.dqk == 128 && L.dv == 128) return launch_variant<2, 128, 128>(L, stream);
        return ADA_ERR_UNSUPPORTED;
    }
    if (L.elt == 1) {
        if (L.dqk == 128 && L.dv == 128) return launch_variant<1, 128, 128>(L, stream);
        if (L.dqk == 64 && L.dv == 128) return launch_variant<1, 64, 128>(L, stream);
        if (L.dqk == 64 && L.dv == 64) return launch_variant<1, 64, 64>(L, stream);
        return ADA_ERR_UNSUPPORTED;
    }
    if (L.dqk == 128 && L.dv == 128) return launch_variant<0, 128, 128>(L, stream);
    if (L.dqk == 64 && L.dv == 128) return launch_variant<0, 64, 128>(L, stream);
    if (L.dqk == 64 && L.dv == 64) return launch_variant<0, 64, 64>(L, stream);
    return ADA_ERR_UNSUPPORTED;
}

}  // namespace ada
