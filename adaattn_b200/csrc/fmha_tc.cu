// K2: fused attention forward on the sm_100a tensor cores.
//
// Persistent CTAs (one per SM) walk a list of work items; an item is two
// 128-row query tiles of one (b, h). Items are ordered head-major (the tiles
// of one head run side by side, so its K and V stream from L2) and, within a
// head, heavy-first (late tiles have more keys under causal masking); small
// jobs take them in groups of heads, heavy-first across each group. The
// producer warp of each CTA takes the next item from a shared counter
// (dynamic scheduling balances the uneven causal items) and broadcasts it to
// the other roles through a small shared-memory ring; without a counter the
// CTAs stride over the list.
//
// Per item, 128-key blocks of K and V stream through a shared-memory ring
// filled by TMA. S = Q K^T (SS) and O += P V (TS: P read from tensor memory)
// run as tcgen05 MMAs with fp32 accumulators in TMEM; the score block never
// leaves the SM. Warp roles (384 threads, three warpgroups):
//   warps 0-3 / 4-7  softmax for query tile 0 / 1: read S from TMEM (one row
//                    per thread), online softmax in registers, write P (16-bit
//                    or E4M3) over the S columns, rescale O when the running
//                    maximum moves, final normalisation and store.
//   warp 8           TMA producer (Q tiles per item, double buffered; then
//                    K_j, V_j through the ring).
//   warp 9           TMEM allocation and the single-thread MMA issuer.
//   warps 10-11      FP16 heads of bf16 inputs (v_convert): convert each
//                    value block from bf16 to fp16 in place in shared memory
//                    between its TMA load and its P·V; otherwise idle (they
//                    complete the third warpgroup, which hands its registers
//                    to the softmax warpgroups).
// The two query tiles ping-pong: while one tile's softmax runs, the tensor
// core works on the other tile's products. Across items the producer and the
// MMA issuer run ahead, so the next item's first products overlap this item's
// final normalisation and stores.
//
// TMEM columns: S0 [0,128) S1 [128,256) O0 [256,256+DV) O1 [256+DV,256+2DV).
// Barrier phases are tracked by running counters across items. Every wait is
// bounded (ada::mbar_wait); a timeout raises the CTA's abort flag and
// ADA_ERR_TIMEOUT in the status word instead of hanging.
#include "ada_common.cuh"
#include "ada_internal.h"

namespace ada {
namespace {

// Three warpgroups: two softmax warpgroups and one for TMA / MMA (two of its
// warps idle). Launched at 168 registers per thread (the cap for 12 warps);
// the TMA/MMA warpgroup gives registers back and the softmax warpgroups take
// them: 2 * 128 * 208 + 128 * 88 = 384 * 168.
constexpr int kThreadsTc = 384;
constexpr int kLaunchRegs = 168;
constexpr int kSoftmaxRegs = 208;
constexpr int kOtherRegs = 88;
// Threads that read each broadcast work item: the MMA issuer and the 256
// softmax threads.
constexpr int kItemConsumers = 1 + 256;
// Threads of warps 10-11, the value-block converters.
constexpr int kConvThreads = 64;
static_assert(2 * 128 * kSoftmaxRegs + 128 * kOtherRegs <= kThreadsTc * kLaunchRegs,
              "register split exceeds the launch pool");
// Dynamic shared memory budget: 227 KB per CTA minus alignment slack and the
// barrier block.
constexpr int kSmemBudget = 232448 - 1024 - 512;
// Split-P scale for fp32 heads: P <= 2^8 under the stale-maximum rule, so
// P * 2^7 stays inside fp16's range and its low part stays normal longer.
constexpr float kSplitPScale = 128.f;
// log2(448): E4M3 P is e4m3(448 * p) with p <= 1 under the exact running maximum.
constexpr float kLog2E4m3Max = 8.807354922057604f;

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
    static constexpr int Q_BYTES = BM * DQK * EB;         // one query tile
    static constexpr int QBUF_BYTES = 2 * Q_BYTES;        // both tiles of one item
    static constexpr int K_BYTES = BN * DQK * EB;
    static constexpr int V_BYTES = BN * DV * EB;
    static constexpr int STAGE_BYTES = K_BYTES > V_BYTES ? K_BYTES : V_BYTES;
    static constexpr int NSTAGE_RAW = (kSmemBudget - 2 * QBUF_BYTES) / STAGE_BYTES;
    static constexpr int NSTAGE = NSTAGE_RAW > 8 ? 8 : NSTAGE_RAW;
    static_assert(NSTAGE >= 2, "ring too small");
    static constexpr int MMA_K = (ELT == 2) ? 32 : 16;   // elements per MMA k-step
    // ELT 3 / 4: FP32 heads of 16-bit inputs. q, k (or q_low, k_low, rounded
    // to the inputs' dtype by the projection) are read as fp16 (3) or bf16 (4)
    // -- in place, or scaled by powers of two into fp16 -- so Q·Kᵀ products
    // are exact and only the fp32 accumulation rounds; v is scaled into fp16
    // (exact) and P keeps fp32 accuracy as an fp16 sum hi + lo (TMEM columns
    // 0..63 and 64..127 of S), each part multiplied into V.
    static constexpr bool SPLIT = ELT == 3 || ELT == 4;
    static_assert(!SPLIT || DV == 128, "split operands: 128-column v rows");
    static constexpr int KSTEP_BYTES = MMA_K * EB;        // 32 bytes either way
    static constexpr int P_COLS = BN * EB / 4;            // TMEM columns holding P
    static constexpr uint32_t FMT = (ELT == 1) ? 1u : 0u; // P·V operands: bf16 = 1, f16 = 0, e4m3 = 0
    // ELT 5: FP16 heads of bf16 inputs. Q·Kᵀ reads the bf16 q, k in place (a
    // bf16 value in fp16's normal range is exactly its fp16 cast, and every
    // product is exact in the fp32 accumulator); P and V (cast) are fp16.
    static constexpr uint32_t FMT_QK = (ELT == 1 || ELT == 4 || ELT == 5) ? 1u : 0u;  // Q·Kᵀ operands
    static constexpr uint32_t IDESC_QK = make_idesc(FMT_QK, FMT_QK, 0, 0, 128, BN);
    static constexpr uint32_t IDESC_PV = make_idesc(FMT, FMT, 0, 1, 128, DV);
    static constexpr int SMEM_BYTES = 2 * QBUF_BYTES + NSTAGE * STAGE_BYTES + 1024 + 512;
};

struct __align__(8) TcBarriers {
    uint64_t q_full[2];
    uint64_t q_empty[2];
    uint64_t s_full[2];
    uint64_t p_full[2];
    uint64_t o_full[2];
    uint64_t teardown;
    uint64_t item_full[4];   // work-item broadcast ring (producer -> consumers)
    uint64_t item_empty[4];
    int64_t item_q[4];
    uint64_t kv_full[8];
    uint64_t kv_empty[8];
    uint64_t v_ready[8];     // value block converted to fp16 (v_convert)
    uint32_t tmem_base;
    int abort_flag;
};

// One work item: the (b, h) slice and the pair of query tiles, with the
// number of key blocks each tile needs.
struct Item {
    int64_t bh;
    int b, h, qtp;
    int n_t[2];
    int nblk;
};

__device__ __forceinline__ int ceil_div_i(int64_t a, int64_t b) { return static_cast<int>((a + b - 1) / b); }

// The n-th item the CTAs take -> its head-major index (what the roles
// broadcast and decode). With head_group G > 1 (jobs of under 8 items per
// SM), heads are taken G at a time, heaviest query-tile pair first across
// the group's heads, so the CTAs that take a launch's last items get light
// ones and finish together (B1 H32 N4096 causal: 667-704 -> 827-910 TFLOP/s);
// with G = 1 the order is head-major, whose K/V reuse in L2 suits larger jobs.
__device__ __forceinline__ int64_t scheduled_item(const TcLaunch& L, int64_t n, int n_qtp) {
    const int G = L.head_group;
    if (G == 1) return n;
    const int bhn = static_cast<int>(L.B * L.H);  // G > 1 only for jobs of under 8 items per SM
    const int n32 = static_cast<int>(n);
    const int grp = n32 / (G * n_qtp);
    const int within = n32 - grp * G * n_qtp;
    const int gsize = (bhn - grp * G) < G ? (bhn - grp * G) : G;
    const int bh = grp * G + within % gsize;
    const int rank = within / gsize;  // 0 = the head's heaviest pair
    return static_cast<int64_t>(bh) * n_qtp + rank;
}

// Head-major work item `it` -> (head, query-tile pair), heaviest pair first
// within each head (under causal masking the late pairs have the most keys).
__device__ __forceinline__ Item decode_item(const TcLaunch& L, int64_t it, int n_qtp, int nkb) {
    Item w;
    w.bh = it / n_qtp;
    w.qtp = n_qtp - 1 - static_cast<int>(it % n_qtp);
    w.b = static_cast<int>(w.bh / L.H);
    w.h = static_cast<int>(w.bh % L.H);
#pragma unroll
    for (int t = 0; t < 2; ++t) {
        const int64_t r0 = (static_cast<int64_t>(w.qtp) * 2 + t) * 128;
        if (r0 >= L.Nq) {
            w.n_t[t] = 0;
        } else if (L.causal) {
            const int64_t r_last = (r0 + 127 < L.Nq - 1) ? r0 + 127 : L.Nq - 1;
            const int need = static_cast<int>(r_last / 128) + 1;
            w.n_t[t] = need < nkb ? need : nkb;
        } else {
            w.n_t[t] = nkb;
        }
    }
    w.nblk = w.n_t[0] > w.n_t[1] ? w.n_t[0] : w.n_t[1];
    return w;
}

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

// The producer picks the CTA's next work item this launch serves: from the
// shared counter (dynamic: a CTA that finishes early takes more items, which
// balances the uneven causal items), or by striding over the list when no
// counter is given. Returns -1 when the list is exhausted.
__device__ __forceinline__ int64_t next_item(const TcLaunch& L, int64_t& static_next, int64_t n_items,
                                             int n_qtp, int nkb) {
    while (true) {
        int64_t it;
        if (L.work_counter != nullptr) {
            it = atomicAdd(L.work_counter, 1);
        } else {
            it = static_next;
            static_next += gridDim.x;
        }
        if (it >= n_items) return -1;
        it = scheduled_item(L, it, n_qtp);
        const Item w = decode_item(L, it, n_qtp, nkb);
        if (head_selected(L.sel, w.bh) && w.nblk > 0) return it;
    }
}

// Consumers read the producer's item choices in order from a 4-slot ring.
__device__ __forceinline__ bool take_item(TcBarriers* bars, uint32_t& ic, int64_t& it,
                                          volatile int* abort_flag, uint64_t tmo, unsigned int* status) {
    const uint32_t slot = ic & 3u;
    if (!mbar_wait(smem_u32(&bars->item_full[slot]), (ic >> 2) & 1u, abort_flag, tmo, status)) return false;
    it = static_cast<const volatile int64_t*>(bars->item_q)[slot];
    mbar_arrive(smem_u32(&bars->item_empty[slot]));
    ++ic;
    return it >= 0;
}

template <int ELT, int DQK, int DV>
__global__ void __launch_bounds__(kThreadsTc, 1) fmha_tc_kernel(const __grid_constant__ TcLaunch L) {
    using C = TcCfg<ELT, DQK, DV>;
    extern __shared__ uint8_t smem_raw[];

    const int n_qt = ceil_div_i(L.Nq, 128);
    const int n_qtp = (n_qt + 1) / 2;
    const int nkb = ceil_div_i(L.Nk, 128);
    const int64_t n_items = L.B * L.H * n_qtp;

    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = base;                        // [2 buffers][2 tiles][Q_BYTES]
    uint8_t* sKV = base + 2 * C::QBUF_BYTES;   // [NSTAGE][STAGE_BYTES]
    TcBarriers* bars = reinterpret_cast<TcBarriers*>(sKV + C::NSTAGE * C::STAGE_BYTES);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // bf16 value blocks converted to fp16 in shared memory (FP16 P·V variants only).
    const bool vconv = (ELT == 0 || ELT == 5) && L.v_convert != 0;

    // A launch for a branch and precision that no head chose ends here,
    // before any setup (the adaptive path launches every variant it may need).
    if (L.sel.decisions != nullptr) {
        int any = 0;
        for (int64_t bh = threadIdx.x; bh < L.B * L.H && !any; bh += blockDim.x) any = head_selected(L.sel, bh);
        if (!__syncthreads_or(any)) return;
    }

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(smem_u32(&bars->q_full[i]), 1);
            // With a staged epilogue each softmax warpgroup also releases the
            // Q buffer after its output tile has left it.
            mbar_init(smem_u32(&bars->q_empty[i]), L.tma_out ? 3 : 1);
            mbar_init(smem_u32(&bars->s_full[i]), 1);
            mbar_init(smem_u32(&bars->p_full[i]), 128);
            mbar_init(smem_u32(&bars->o_full[i]), 1);
        }
        mbar_init(smem_u32(&bars->teardown), 1);
        for (int i = 0; i < 4; ++i) {
            mbar_init(smem_u32(&bars->item_full[i]), 1);
            mbar_init(smem_u32(&bars->item_empty[i]), kItemConsumers + (vconv ? kConvThreads : 0));
        }
        for (int s = 0; s < C::NSTAGE; ++s) {
            mbar_init(smem_u32(&bars->kv_full[s]), 1);
            mbar_init(smem_u32(&bars->kv_empty[s]), 1);
            mbar_init(smem_u32(&bars->v_ready[s]), kConvThreads);
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
    // Launch fields read inside the loops are copied to registers: the asm
    // memory clobbers of the barrier and tensor-memory wrappers would
    // otherwise make every use reload them from parameter space.
    unsigned int* const status = L.status;

    if (warp >= 8) {
      regs_decrease<kOtherRegs>();
      if (warp == 8) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            tma_prefetch_desc(&L.tq);
            tma_prefetch_desc(&L.tk);
            tma_prefetch_desc(&L.tv);
            uint32_t qi = 0;   // items loaded by this CTA
            uint32_t kvi = 0;  // ring slots filled
            uint32_t ic = 0;   // items broadcast
            int64_t static_next = blockIdx.x;
            bool ok = true;
            while (ok) {
                const int64_t it = next_item(L, static_next, n_items, n_qtp, nkb);
                const uint32_t slot = ic & 3u;
                ok = mbar_wait(smem_u32(&bars->item_empty[slot]), ((ic >> 2) & 1u) ^ 1u, abort_flag, tmo,
                               status);
                if (!ok) break;
                static_cast<volatile int64_t*>(bars->item_q)[slot] = it;
                mbar_arrive(smem_u32(&bars->item_full[slot]));
                ++ic;
                if (it < 0) break;
                const Item w = decode_item(L, it, n_qtp, nkb);
                const uint32_t qb = qi & 1u;
                ok = mbar_wait(smem_u32(&bars->q_empty[qb]), ((qi >> 1) & 1u) ^ 1u, abort_flag, tmo, status);
                if (!ok) break;
                const uint32_t qbar = smem_u32(&bars->q_full[qb]);
                mbar_arrive_expect_tx(qbar, C::QBUF_BYTES);
                for (int t = 0; t < 2; ++t)
                    for (int a = 0; a < C::QK_ATOMS; ++a)
                        tma_load_4d(smem_u32(sQ + qb * C::QBUF_BYTES + t * C::Q_BYTES + a * C::BOX), &L.tq,
                                    qbar, a * C::ATOM_COLS, (w.qtp * 2 + t) * 128, w.h, w.b);
                ++qi;
                for (int j = 0; ok && j < w.nblk; ++j) {
                    for (int half = 0; half < 2; ++half) {
                        const uint32_t st = kvi % C::NSTAGE;
                        const uint32_t ph = (kvi / C::NSTAGE) & 1u;
                        ok = mbar_wait(smem_u32(&bars->kv_empty[st]), ph ^ 1u, abort_flag, tmo, status);
                        if (!ok) break;
                        const uint32_t fbar = smem_u32(&bars->kv_full[st]);
                        uint8_t* dst = sKV + st * C::STAGE_BYTES;
                        if (half == 0) {
                            mbar_arrive_expect_tx(fbar, C::K_BYTES);
                            for (int a = 0; a < C::QK_ATOMS; ++a)
                                tma_load_4d(smem_u32(dst + a * C::BOX), &L.tk, fbar, a * C::ATOM_COLS,
                                            j * 128, w.h, w.b);
                        } else {
                            mbar_arrive_expect_tx(fbar, C::V_BYTES);
                            for (int a = 0; a < C::V_ATOMS; ++a)
                                tma_load_4d(smem_u32(dst + a * C::BOX), &L.tv, fbar, a * C::ATOM_COLS,
                                            j * 128, w.h, w.b);
                        }
                        ++kvi;
                    }
                }
            }
        }
        __syncwarp();
    } else if (warp == 9) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t sQa = smem_u32(sQ);
            const uint32_t sKVa = smem_u32(sKV);
            uint32_t qi = 0, kvi = 0, ic = 0;
            uint32_t pc[2] = {0u, 0u};  // P blocks consumed per tile
            uint32_t vpar = 0;          // per ring slot: parity of its v_ready phase
            bool ok = true;
            int64_t it;
            auto issue_s = [&](int t, uint32_t qbuf, uint32_t stage) {
                const uint32_t q0 = sQa + qbuf * C::QBUF_BYTES + t * C::Q_BYTES;
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
            auto issue_pv = [&](int t, uint32_t stage, bool first) {
                const uint32_t v0 = sKVa + stage * C::STAGE_BYTES;
#pragma unroll
                for (int part = 0; part < (C::SPLIT ? 2 : 1); ++part) {
#pragma unroll
                    for (int ks = 0; ks < C::BN / C::MMA_K; ++ks) {
                        const uint64_t bd = make_sdesc_sw128(v0 + ks * C::MMA_K * 128, C::BOX, 1024);
                        const uint32_t a_t = tmem + t * 128 + part * 64 + ks * (C::MMA_K * C::EB / 4);
                        issue_mma_ts<ELT>(tmem + 256 + t * DV, a_t, bd, C::IDESC_PV,
                                          (!first || part > 0 || ks > 0) ? 1u : 0u);
                    }
                }
            };
            while (ok && take_item(bars, ic, it, abort_flag, tmo, status)) {
                const Item w = decode_item(L, it, n_qtp, nkb);
                const uint32_t qb = qi & 1u;
                ok = mbar_wait(smem_u32(&bars->q_full[qb]), (qi >> 1) & 1u, abort_flag, tmo, status);
                if (!ok) break;
                // K_0 and the first score blocks.
                {
                    const uint32_t st = kvi % C::NSTAGE;
                    ok = mbar_wait(smem_u32(&bars->kv_full[st]), (kvi / C::NSTAGE) & 1u, abort_flag, tmo, status);
                    if (!ok) break;
                    tc_fence_after();
                    for (int t = 0; t < 2; ++t)
                        if (w.n_t[t] > 0) issue_s(t, qb, st);
                    tc_commit(smem_u32(&bars->kv_empty[st]));
                }
                for (int j = 0; ok && j < w.nblk; ++j) {
                    const uint32_t iv = kvi + 2 * j + 1;
                    const uint32_t sv = iv % C::NSTAGE;
                    // v_ready completes only for the value blocks of a slot (a slot
                    // also takes key blocks when the ring length is odd): its
                    // parity is tracked per slot.
                    const uint32_t vph = vconv ? ((vpar >> sv) & 1u) : ((iv / C::NSTAGE) & 1u);
                    ok = mbar_wait(smem_u32(vconv ? &bars->v_ready[sv] : &bars->kv_full[sv]), vph, abort_flag, tmo,
                                   status);
                    vpar ^= vconv ? (1u << sv) : 0u;
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t ik = kvi + 2 * j + 2;
                    const uint32_t sk = ik % C::NSTAGE;
                    bool k_ready = false;
#pragma unroll
                    for (int t = 0; t < 2; ++t) {
                        if (!ok) break;
                        if (j < w.n_t[t]) {
                            ok = mbar_wait(smem_u32(&bars->p_full[t]), pc[t] & 1u, abort_flag, tmo, status);
                            if (!ok) break;
                            ++pc[t];
                            tc_fence_after();
                            issue_pv(t, sv, j == 0);
                            if (j == w.n_t[t] - 1) tc_commit(smem_u32(&bars->o_full[t]));
                        }
                        if (j + 1 < w.n_t[t]) {
                            if (!k_ready) {
                                ok = mbar_wait(smem_u32(&bars->kv_full[sk]), (ik / C::NSTAGE) & 1u,
                                               abort_flag, tmo, status);
                                if (!ok) break;
                                tc_fence_after();
                                k_ready = true;
                            }
                            issue_s(t, qb, sk);
                        }
                    }
                    tc_commit(smem_u32(&bars->kv_empty[sv]));
                    if (k_ready) tc_commit(smem_u32(&bars->kv_empty[sk]));
                }
                // Every S product of this item is issued: the Q buffer frees
                // when they complete.
                tc_commit(smem_u32(&bars->q_empty[qb]));
                kvi += 2 * w.nblk;
                ++qi;
            }
            // Everything issued so far completes before the CTA frees TMEM.
            tc_commit(smem_u32(&bars->teardown));
            teardown_wait(smem_u32(&bars->teardown), 0, tmo, status);
        }
        __syncwarp();
      } else if (vconv) {
        // ---------------- value-block converters (warps 10-11) ----------------
        // Each value block, once TMA has landed it, is rewritten in place as
        // fp16 (same positions in the swizzled layout: the conversion is
        // elementwise), then handed to the MMA issuer. Rounding: round to
        // nearest, overflow to infinity, as a cast of v to fp16 does.
        if constexpr (ELT == 0 || ELT == 5) {
            const int ct = static_cast<int>(threadIdx.x) - 320;
            uint32_t ic = 0, kvi = 0;
            bool ok = true;
            int64_t it;
            while (ok && take_item(bars, ic, it, abort_flag, tmo, status)) {
                const Item w = decode_item(L, it, n_qtp, nkb);
                for (int j = 0; ok && j < w.nblk; ++j) {
                    const uint32_t iv = kvi + 2 * j + 1;
                    const uint32_t sv = iv % C::NSTAGE;
                    ok = mbar_wait(smem_u32(&bars->kv_full[sv]), (iv / C::NSTAGE) & 1u, abort_flag, tmo, status);
                    if (!ok) break;
                    uint4* blk = reinterpret_cast<uint4*>(sKV + sv * C::STAGE_BYTES);
#pragma unroll 4
                    for (int c = ct; c < C::V_BYTES / 16; c += kConvThreads) {
                        const uint4 x = blk[c];
                        const uint32_t wi[4] = {x.x, x.y, x.z, x.w};
                        uint32_t wo[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e)
                            wo[e] = pack_f16x2(__uint_as_float(wi[e] << 16), __uint_as_float(wi[e] & 0xFFFF0000u));
                        blk[c] = make_uint4(wo[0], wo[1], wo[2], wo[3]);
                    }
                    // The tensor core reads the block through the async proxy.
                    fence_proxy_async_smem();
                    mbar_arrive(smem_u32(&bars->v_ready[sv]));
                }
                kvi += 2 * w.nblk;
            }
        }
      }
    } else {
        regs_increase<kSoftmaxRegs>();
        const float scale_log2 = L.scale_log2;
        const bool causal = L.causal != 0;
        const void* const mask_data = L.mask.data;
        const int round_dtype = L.round_dtype, out_dtype = L.out_dtype, out_vec = L.out_vec;
        const int dv_out = L.dv_out;
        const bool tma_out = L.tma_out != 0;
        // ---------------- softmax warpgroups ----------------
        const int t = warp >> 2;
        const int row = (warp & 3) * 32 + lane;  // TMEM lane == row of the tile
        const uint32_t lane_bits = static_cast<uint32_t>((warp & 3) * 32) << 16;
        const uint32_t tS = tmem + lane_bits + t * 128;
        const uint32_t tO = tmem + lane_bits + 256 + t * DV;
        uint32_t sc = 0;  // S blocks consumed by this tile
        uint32_t oc = 0;  // items finished by this tile
        bool ok = true;
        uint32_t ic = 0;
        uint32_t qn = 0;  // items seen: the item's Q buffer is qn & 1
        const bool leader = (threadIdx.x & 127) == 0;
        int64_t it;
        while (ok && take_item(bars, ic, it, abort_flag, tmo, status)) {
            const Item w = decode_item(L, it, n_qtp, nkb);
            const int nt = w.n_t[t];
            const uint32_t qb = qn & 1u;
            ++qn;
            if (nt == 0) {
                if (tma_out && leader) mbar_arrive(smem_u32(&bars->q_empty[qb]));
                continue;
            }
            const int tile_r0 = (w.qtp * 2 + t) * 128;
            const int qrow = tile_r0 + row;
            const int Nk = static_cast<int>(L.Nk);
            float sq = 1.f;
            if constexpr (ELT >= 2 && ELT <= 4)
                if (L.q_scale != nullptr) sq = L.q_scale[w.bh * L.nt_q + (w.qtp * 2 + t)];
            float m_run = -INFINITY;
            float l_run = 0.f;
            for (int j = 0; j < nt; ++j) {
                // The key tile's scale is loaded before the wait for S, off
                // the softmax's critical path.
                float ksc = 1.f;
                if constexpr (ELT >= 2 && ELT <= 4)
                    if (L.k_scale != nullptr) ksc = L.k_scale[w.bh * L.nt_k + j];
                ok = mbar_wait(smem_u32(&bars->s_full[t]), sc & 1u, abort_flag, tmo, status);
                if (!ok) break;
                ++sc;
                tc_fence_after();
                float s[128];
                {
                    uint32_t r0[32], r1[32], r2[32], r3[32];
                    tmem_ld32(tS + 0, r0);
                    tmem_ld32(tS + 32, r1);
                    tmem_ld32(tS + 64, r2);
                    tmem_ld32(tS + 96, r3);
                    tmem_ld_wait();
                    reg_fence32(r0);
                    reg_fence32(r1);
                    reg_fence32(r2);
                    reg_fence32(r3);
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        s[i] = __uint_as_float(r0[i]);
                        s[32 + i] = __uint_as_float(r1[i]);
                        s[64 + i] = __uint_as_float(r2[i]);
                        s[96 + i] = __uint_as_float(r3[i]);
                    }
                }
                float sl2 = scale_log2;
                if constexpr (ELT >= 2 && ELT <= 4)
                    if (L.k_scale != nullptr) sl2 *= sq * ksc;
                const int kv0 = j * 128;
                const bool edge = (kv0 + 128 > Nk) || (causal && kv0 + 127 > tile_r0);
                if (edge) {
                    const int lim_k = Nk - kv0;                                   // keys >= Nk
                    const int lim_c = causal ? (qrow - kv0 + 1) : 128;          // keys > qrow
                    const int lim = lim_k < lim_c ? lim_k : lim_c;
#pragma unroll
                    for (int c = 0; c < 128; ++c)
                        if (c >= lim) s[c] = -INFINITY;
                }
                if (mask_data != nullptr && qrow < L.Nq) {
                    // logits are s * scale + m; in raw-score units that is s + m / scale.
                    const float inv_scale = 1.f / (sl2 * 0.69314718056f);
                    const int64_t mb = w.b * L.mask.s[0] + w.h * L.mask.s[1] + qrow * L.mask.s[2];
#pragma unroll
                    for (int c = 0; c < 128; ++c) {
                        const int kv = kv0 + c;
                        if (kv < Nk) {
                            const float mv = load_as_f32(mask_data, mb + kv * L.mask.s[3], L.mask.dtype);
                            if (L.mask.dtype == ADA_BOOL) {
                                if (mv == 0.f) s[c] = -INFINITY;
                            } else {
                                s[c] += round_to(mv, round_dtype) * inv_scale;
                            }
                        }
                    }
                }
                // Row maximum: 8 chains over s[0..127] (two new values per
                // three-input max, the last eight with a plain max).
                float mx[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) mx[i] = s[i];
#pragma unroll
                for (int c = 8; c + 16 <= 128; c += 16)
#pragma unroll
                    for (int i = 0; i < 8; ++i) mx[i] = max3f(mx[i], s[c + i], s[c + 8 + i]);
#pragma unroll
                for (int i = 0; i < 8; ++i) mx[i] = fmaxf(mx[i], s[120 + i]);
                const float m_blk = max3f(max3f(mx[0], mx[1], mx[2]), max3f(mx[3], mx[4], mx[5]),
                                          fmaxf(mx[6], mx[7]));
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
                // E4M3 P is quantised as e4m3(448 * p): the factor 448 rides
                // in the exponent (2^(x + log2 448)), and l sums 448 * p.
                const float neg_m = (m_new == -INFINITY) ? 0.f : (ELT == 2 ? kLog2E4m3Max - m_new : -m_new);
                const uint64_t sl2p = f2_pack(sl2, sl2);
                const uint64_t nmp = f2_pack(neg_m, neg_m);
                uint64_t ls0 = f2_pack(0.f, 0.f), ls1 = ls0;
                // P = 2^(s * scale * log2(e) - m), written over the S columns.
                {
                    constexpr int NP = C::P_COLS / 32;  // 32-column chunks of P
                    uint32_t pr[32];
                    if constexpr (C::SPLIT) {
                        // P * 2^7 = hi + lo, both fp16 (hi <= 2^15); hi over
                        // S columns 0..63, lo over 64..127, 16 columns at a time.
#pragma unroll
                        for (int q16 = 0; q16 < 4; ++q16) {
                            uint32_t ph[16], pl[16];
#pragma unroll
                            for (int i = 0; i < 16; ++i) {
                                const int c = q16 * 32 + i * 2;
                                float p0, p1;
                                f2_unpack(f2_fma(f2_pack(s[c], s[c + 1]), sl2p, nmp), p0, p1);
                                p0 = fast_exp2(p0);
                                p1 = fast_exp2(p1);
                                if (i & 1)
                                    ls1 = f2_add(ls1, f2_pack(p0, p1));
                                else
                                    ls0 = f2_add(ls0, f2_pack(p0, p1));
                                const float h0 = p0 * kSplitPScale, h1 = p1 * kSplitPScale;
                                ph[i] = pack_f16x2(h0, h1);
                                float r0, r1;
                                unpack_f16x2(ph[i], r0, r1);
                                pl[i] = pack_f16x2(h0 - r0, h1 - r1);
                            }
                            tmem_st16(tS + q16 * 16, ph);
                            tmem_st16(tS + 64 + q16 * 16, pl);
                        }
                    }
#pragma unroll
                    for (int chunk = 0; chunk < (C::SPLIT ? 0 : NP); ++chunk) {
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            if constexpr (ELT == 2) {
                                const int c = chunk * 128 + i * 4;
                                float p0, p1, p2, p3;
                                f2_unpack(f2_fma(f2_pack(s[c], s[c + 1]), sl2p, nmp), p0, p1);
                                f2_unpack(f2_fma(f2_pack(s[c + 2], s[c + 3]), sl2p, nmp), p2, p3);
                                p0 = fast_exp2(p0);
                                p1 = fast_exp2(p1);
                                p2 = fast_exp2(p2);
                                p3 = fast_exp2(p3);
                                ls0 = f2_add(ls0, f2_pack(p0, p1));
                                ls1 = f2_add(ls1, f2_pack(p2, p3));
                                pr[i] = pack_e4m3x4(p0, p1, p2, p3);
                            } else {
                                const int c = chunk * 64 + i * 2;
                                float p0, p1;
                                f2_unpack(f2_fma(f2_pack(s[c], s[c + 1]), sl2p, nmp), p0, p1);
                                p0 = fast_exp2(p0);
                                p1 = fast_exp2(p1);
                                if (i & 1)
                                    ls1 = f2_add(ls1, f2_pack(p0, p1));
                                else
                                    ls0 = f2_add(ls0, f2_pack(p0, p1));
                                pr[i] = (ELT == 1) ? pack_bf16x2(p0, p1) : pack_f16x2(p0, p1);
                            }
                        }
                        tmem_st32(tS + chunk * 32, pr);
                    }
                }
                float la, lb, lc, ld;
                f2_unpack(ls0, la, lb);
                f2_unpack(ls1, lc, ld);
                l_run = l_run * alpha + ((la + lb) + (lc + ld));
                if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
                    const uint64_t ap = f2_pack(alpha, alpha);
                    uint32_t r[32];
#pragma unroll
                    for (int c = 0; c < DV / 32; ++c) {
                        tmem_ld32(tO + c * 32, r);
                        tmem_ld_wait();
                        reg_fence32(r);
#pragma unroll
                        for (int i = 0; i < 32; i += 2) {
                            float x0, x1;
                            f2_unpack(f2_mul(f2_pack(__uint_as_float(r[i]), __uint_as_float(r[i + 1])), ap), x0, x1);
                            r[i] = __float_as_uint(x0);
                            r[i + 1] = __float_as_uint(x1);
                        }
                        tmem_st32(tO + c * 32, r);
                    }
                }
                m_run = m_new;
                tmem_st_wait();
                tc_fence_before();
                mbar_arrive(smem_u32(&bars->p_full[t]));
            }
            if (!ok) break;
            ok = mbar_wait(smem_u32(&bars->o_full[t]), oc & 1u, abort_flag, tmo, status);
            if (!ok) break;
            ++oc;
            tc_fence_after();
            // ---- epilogue: O / l, rounded like the reference's result, stored ----
            float post = 1.f / l_run;
            if constexpr (ELT == 2) post *= L.v_scale[w.bh];  // l_run already carries the factor 448
            if constexpr (C::SPLIT) post *= L.v_scale[w.bh] * (1.f / kSplitPScale);
            const bool row_ok = qrow < L.Nq;
            uint8_t* orow = reinterpret_cast<uint8_t*>(L.out);
            const int64_t obase = w.b * L.os[0] + w.h * L.os[1] + static_cast<int64_t>(qrow) * L.os[2];
            // The reference's result is rounded to its compute dtype before the
            // cast to the output dtype; when the two agree the packing below
            // is that rounding.
            const bool pre_round = round_dtype != out_dtype && round_dtype != ADA_F32;
            uint32_t r[32];
            if constexpr (ELT != 2 && DQK == 128 && DV == 128) {
                if (tma_out) {
                    // Stage the 16-bit tile in this tile's Q slot (no longer read:
                    // every Q K^T of the item has completed) in the 128-byte
                    // swizzled box layout, then one thread stores it with TMA.
                    uint8_t* stg = sQ + qb * C::QBUF_BYTES + t * C::Q_BYTES;
#pragma unroll
                    for (int c = 0; c < DV / 32; ++c) {
                        tmem_ld32(tO + c * 32, r);
                        tmem_ld_wait();
                        reg_fence32(r);
                        uint32_t wv[16];
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            float x0 = __uint_as_float(r[2 * i]) * post, x1 = __uint_as_float(r[2 * i + 1]) * post;
                            if (pre_round) {
                                x0 = round_to(x0, round_dtype);
                                x1 = round_to(x1, round_dtype);
                            }
                            wv[i] = (out_dtype == ADA_BF16) ? pack_bf16x2(x0, x1) : pack_f16x2(x0, x1);
                        }
                        const int atom = (c * 32) / 64;
                        uint8_t* line = stg + atom * C::BOX + row * 128;
#pragma unroll
                        for (int k4 = 0; k4 < 4; ++k4) {
                            const int chunk = ((c * 32) % 64) / 8 + k4;  // 16-byte chunk within the line
                            *reinterpret_cast<uint4*>(line + ((chunk ^ (row & 7)) * 16)) =
                                make_uint4(wv[4 * k4], wv[4 * k4 + 1], wv[4 * k4 + 2], wv[4 * k4 + 3]);
                        }
                    }
                    fence_proxy_async_smem();
                    if (t == 0)
                        named_barrier_sync(1, 128);
                    else
                        named_barrier_sync(2, 128);
                    if (leader) {
                        for (int a = 0; a * 64 < dv_out && a < DV / 64; ++a)
                            tma_store_4d(&L.to, smem_u32(stg + a * C::BOX), a * 64, tile_r0, w.h, w.b);
                        bulk_commit_group();
                        bulk_wait_group_read0();
                        mbar_arrive(smem_u32(&bars->q_empty[qb]));
                    }
                    continue;
                }
            }
#pragma unroll
            for (int c = 0; c < DV / 32; ++c) {
                tmem_ld32(tO + c * 32, r);
                tmem_ld_wait();
                reg_fence32(r);
                if (row_ok) {
                    float o[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const float x = __uint_as_float(r[i]) * post;
                        o[i] = pre_round ? round_to(x, round_dtype) : x;
                    }
                    const int col0 = c * 32;
                    if (out_vec && col0 + 32 <= dv_out) {
                        if (out_dtype == ADA_F32) {
                            if (out_vec == 32) {
#pragma unroll
                                for (int i = 0; i < 4; ++i)
                                    st_global_v8(orow + (obase + col0 + 8 * i) * 4,
                                                 reinterpret_cast<const uint32_t*>(o + 8 * i));
                            } else {
                                float4* dst = reinterpret_cast<float4*>(orow + (obase + col0) * 4);
#pragma unroll
                                for (int i = 0; i < 8; ++i)
                                    dst[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
                            }
                        } else {
                            uint32_t wv[16];
                            if (out_dtype == ADA_BF16) {
#pragma unroll
                                for (int i = 0; i < 16; ++i) wv[i] = pack_bf16x2(o[2 * i], o[2 * i + 1]);
                            } else {
#pragma unroll
                                for (int i = 0; i < 16; ++i) wv[i] = pack_f16x2(o[2 * i], o[2 * i + 1]);
                            }
                            uint8_t* dst = orow + (obase + col0) * 2;
                            if (out_vec == 32) {
                                st_global_v8(dst, wv);
                                st_global_v8(dst + 32, wv + 8);
                            } else {
#pragma unroll
                                for (int i = 0; i < 4; ++i)
                                    reinterpret_cast<uint4*>(dst)[i] =
                                        make_uint4(wv[4 * i], wv[4 * i + 1], wv[4 * i + 2], wv[4 * i + 3]);
                            }
                        }
                    } else {
                        for (int i = 0; i < 32; ++i)
                            if (col0 + i < dv_out)
                                store_from_f32(L.out, obase + (col0 + i) * L.os[3], out_dtype, o[i]);
                    }
                }
            }
        }
    }

    // Output tiles stored with TMA are complete before the CTA exits.
    if (L.tma_out && warp < 8 && (threadIdx.x & 127) == 0) bulk_wait_group0();
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
    // The register hand-over inside the kernel needs the full launch pool; a
    // build that allocated fewer registers would wait forever in setmaxnreg.
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, kern) != cudaSuccess || fa.numRegs != kLaunchRegs)
        return ADA_ERR_UNSUPPORTED;
    const int64_t n_qt = (L.Nq + 127) / 128;
    const int64_t n_qtp = (n_qt + 1) / 2;
    const int64_t items = n_qtp * L.B * L.H;
    if (items <= 0) return ADA_OK;
    if (L.head_group < 1) return ADA_ERR_INVALID;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return ADA_ERR_LAUNCH;
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
        return ADA_ERR_LAUNCH;
    const int64_t grid = items < sms ? items : sms;
    kern<<<static_cast<unsigned>(grid), kThreadsTc, C::SMEM_BYTES, stream>>>(L);
    return cudaGetLastError() == cudaSuccess ? ADA_OK : ADA_ERR_LAUNCH;
}

}  // namespace

int launch_fmha_tc(const TcLaunch& L, cudaStream_t stream) {
    if (L.elt == 3) {
        if (L.dqk == 128 && L.dv == 128) return launch_variant<3, 128, 128>(L, stream);
        if (L.dqk == 64 && L.dv == 128) return launch_variant<3, 64, 128>(L, stream);
        return ADA_ERR_UNSUPPORTED;
    }
    if (L.elt == 4) {
        if (L.dqk == 128 && L.dv == 128) return launch_variant<4, 128, 128>(L, stream);
        if (L.dqk == 64 && L.dv == 128) return launch_variant<4, 64, 128>(L, stream);
        return ADA_ERR_UNSUPPORTED;
    }
    if (L.elt == 5) {
        if (L.dqk == 128 && L.dv == 128) return launch_variant<5, 128, 128>(L, stream);
        if (L.dqk == 64 && L.dv == 128) return launch_variant<5, 64, 128>(L, stream);
        if (L.dqk == 64 && L.dv == 64) return launch_variant<5, 64, 64>(L, stream);
        return ADA_ERR_UNSUPPORTED;
    }
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
