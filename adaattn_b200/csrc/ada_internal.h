// Host-side launch interfaces shared by the kernel files and the C ABI layer.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/adaattn_b200.h"

namespace ada {

// --- analyzer ---------------------------------------------------------------
struct AnalyzeLaunch {
    const void* q;
    const void* k;
    int dtype;
    int64_t B, H, Nq, Nk, D;
    int64_t qs[4], ks[4];
    float scale, eps;
    double log_s;
    int S, stride;
    float* head_stats;
    float* head_sum;
    int32_t* decisions;
    float* summary;
    double rank_threshold;
    int enable_rank, enable_prec, default_prec, allow_fp8, granularity;
    unsigned int* status;  // device status word for the bounded wait of the tensor-core sample product
    uint64_t timeout_ns;
};
int launch_analyze(const AnalyzeLaunch& L, cudaStream_t stream);
int launch_entropy_rows(const void* w, int dtype, int64_t rows, int64_t len, float* out,
                        cudaStream_t stream);
int launch_effective_rank(const void* w, int dtype, int64_t groups, int64_t group, int64_t len,
                          float* out, cudaStream_t stream);
int launch_target_ranks(const float* eff, int64_t n, int64_t min_rank, int64_t max_rank, double thr,
                        int64_t* out, cudaStream_t stream);
int launch_bounded_wait(uint64_t timeout_ns, unsigned int* status, cudaStream_t stream);
// Sets the calling thread's ada_get_last_error message; returns `code`.
int record_last_error(int code, const char* msg);
// The argument checks of the analyzer entry points (device, tensors, shapes,
// dtypes, parameters) and the launch description they imply; head_sum is left
// null for the caller to point at its scratch. Returns ADA_OK or the ADA_ERR_*
// code, with the message recorded for ada_get_last_error.
int analyze_setup(const AdaTensor* q, const AdaTensor* k, const AdaAnalyzeParams* params, int32_t* decisions,
                  float* head_stats, float* summary, AnalyzeLaunch* L);
// Checks for an sm_100 device and resolves its status word (once per device).
int device_status_word(unsigned int** status);
// cuTensorMapEncodeTiled from the driver (resolved once).
int tensor_map_encoder(PFN_cuTensorMapEncodeTiled_v12000* fn);
// Limit of every bounded device-side wait (ADA_WAIT_TIMEOUT_MS, default 4 s).
uint64_t default_wait_timeout_ns();

// --- which heads a launch serves ---------------------------------------------
// A head (b,h) is served when decisions == nullptr (static decision) or when
// its precision code is in prec_mask and its low-rank flag equals low_rank.
struct HeadSelect {
    const int32_t* decisions;
    uint32_t prec_mask;
    int low_rank;
};

__host__ __device__ inline bool head_selected(const HeadSelect& s, int64_t bh) {
#ifdef __CUDA_ARCH__
    if (s.decisions == nullptr) return true;
    const int p = s.decisions[bh * 2 + 0];
    const int l = s.decisions[bh * 2 + 1];
    return ((s.prec_mask >> p) & 1u) && (l != 0) == (s.low_rank != 0);
#else
    (void)s;
    (void)bh;
    return true;
#endif
}

// Optional additive / boolean mask, broadcast view over [B, H, Nq, Nk].
struct MaskView {
    const void* data;  // nullptr: no mask
    int dtype;         // ADA_BOOL or a float type
    int64_t s[4];
};

// --- operand preparation (casts, low-rank projection, E4M3 quantisation) ----
// Where each (b,h) slice's decision comes from.
struct DecisionSrc {
    const int32_t* decisions;  // [B*H*2] or nullptr
    int static_prec, static_low;
};

__host__ __device__ inline void get_decision(const DecisionSrc& d, int64_t bh, int* prec, int* low) {
    if (d.decisions != nullptr) {
        *prec = d.decisions[bh * 2 + 0];
        *low = d.decisions[bh * 2 + 1];
    } else {
        *prec = d.static_prec;
        *low = d.static_low;
    }
}

struct PrepLaunch {
    DecisionSrc dec;
    // inputs [B,H,N,D]
    const void* q;
    const void* k;
    const void* v;
    int in_dtype;
    int64_t B, H, Nq, Nk, D;
    int64_t qs[4], ks[4], vs[4];
    const void* w_down;  // [r, D] row-major contiguous, or nullptr
    int w_dtype;
    int64_t r;
    // 16-bit region: heads of the 16-bit tensor-core precisions that cannot be
    // read in place (dtype change, low rank, or layout) -- [B,H,N,ld]
    uint32_t tc16_mask;   // precision codes served by the 16-bit kernels
    uint32_t f16_mask;    // ...of which these compute in fp16 (the rest bf16)
    int direct_ok;        // dense heads already in their compute dtype are read in place
    int mixed16;          // dense FP16 heads of bf16 inputs read q, k in place: only v is cast
    int v_direct;         // 16-bit heads whose compute dtype is the inputs' (or FP16 of bf16 inputs, converted
                          // in the attention kernel) read v in place: no cast copy of v
    void* ws16_q;
    void* ws16_k;
    void* ws16_v;
    int64_t ld16_qk, ld16_v;
    int dqk_dense, dqk_low, dv_pad;  // padded widths written (zero filled)
    // fp32 region for FP32 low-rank heads: q_low/k_low [B,H,N,r]
    uint32_t fp32_mask;
    float* ws32_q;
    float* ws32_k;
    // e4m3 region [B,H,N,128] plus per-tile scales
    uint32_t fp8_mask;
    uint8_t* ws8_q;
    uint8_t* ws8_k;
    uint8_t* ws8_v;
    float* amax_q;  // [B,H,nt_q]
    float* amax_k;  // [B,H,nt_k]
    float* amax_v;  // [B,H,nt_k]
    float* scale_q; // [B,H,nt_q]
    float* scale_k; // [B,H,nt_k]
    float* scale_v; // [B,H]
    int64_t nt_q, nt_k;
    int low_src16;  // 1: low-rank q_low/k_low are already in the 16-bit region (input dtype)
    // FP32 heads of 16-bit inputs on the tensor cores: q, k (dense heads) or
    // q_low, k_low (low-rank heads with r <= 64, from the fp32 region; values
    // of the inputs' dtype) and v scaled by powers of two into fp16:
    // q, k [B*H][N][split_ld] (64 columns for low rank, dqk_dense for dense
    // heads), v [B*H][N][128].
    uint32_t split_mask;      // precision codes served this way (FP32) or 0
    int split_low, split_dense;  // which FP32 heads (low rank / dense) are served
    int split_qk_low, split_qk_dense;  // 1: their q/k are scaled into wss_q/wss_k (else read in place)
    int64_t split_ld;
    uint16_t* wss_q;
    uint16_t* wss_k;
    uint16_t* wss_v;
    float* split_sq;          // [B,H,nt_q] power-of-two scales of q_low tiles
    float* split_sk;          // [B,H,nt_k]
    float* split_sv;          // [B,H]
    unsigned int* split_amax_v;  // [B,H] max |v| bits, zeroed before launch_split
    unsigned int* status;        // device status word (bounded waits record ADA_ERR_TIMEOUT)
    uint64_t timeout_ns;
};
int launch_prep16(const PrepLaunch& L, cudaStream_t stream);

// Tensor-core projection of q and k for low-rank heads (16-bit inputs,
// D in {64, 128}); outputs as in PrepLaunch's 16-bit / fp32 regions.
struct ProjLaunch {
    CUtensorMap tq, tk;  // [B,H,N,D] inputs, 64-column x 128-row boxes
    CUtensorMap tw;      // rank_proj_down.weight [r, D], 64-column x r_pad-row boxes
    DecisionSrc dec;
    int in_dtype;
    int64_t B, H, Nq, Nk;
    int D, r, r_pad;
    uint32_t tc16_mask, f16_mask, fp32_mask;
    uint32_t in16_mask;  // E4M3 heads and FP32 heads on the tensor cores: q_low/k_low to the 16-bit region in the input dtype
    void* ws16_q;
    void* ws16_k;
    int64_t ld16;
    float* ws32_q;
    float* ws32_k;
    unsigned int* status;
    uint64_t timeout_ns;
    // Output through TMA stores (r_pad 64): 16-bit regions [B*H][N][ld16]
    // (64-column x 128-row boxes) and fp32 regions [B*H][N][r] (32-column boxes).
    int tma16, tma32;
    CUtensorMap to16_q, to16_k, to32_q, to32_k;
};
int launch_proj_tc(const ProjLaunch& L, cudaStream_t stream);
// Vectorised casts for the 16-bit operand region: every tensor of dense heads
// that are cast, only V for low-rank heads (their q, k come from the projection).
int launch_cast16(const PrepLaunch& L, int skip_low_rank_qk, cudaStream_t stream);
int launch_prep32(const PrepLaunch& L, cudaStream_t stream);
int launch_prep8(const PrepLaunch& L, cudaStream_t stream);
int launch_split(const PrepLaunch& L, cudaStream_t stream);

// --- tensor-core FMHA (tcgen05) -----------------------------------------------
struct TcLaunch {
    CUtensorMap tq, tk, tv;
    int elt;          // 0 f16, 1 bf16, 2 e4m3; FP32 heads (P as fp16 hi + lo, fp16 V): 3 fp16 q/k, 4 bf16 q/k;
                      // 5 FP16 heads of bf16 inputs: bf16 q/k in place, fp16 P and V
    int dqk, dv;      // operand widths (64 or 128)
    int v_convert;    // elt 0 / 5 only: 1 = tv maps the bf16 v itself and the kernel converts each
                      // value block to fp16 in shared memory before P·V (no cast copy of v)
    int64_t B, H, Nq, Nk;
    int dv_out;       // real value width stored
    void* out;
    int out_dtype;
    int64_t os[4];
    int out_vec;      // widest aligned vector store for output rows: 32, 16 or 0 bytes
    int tma_out;      // 1: the epilogue stages O in the item's Q slot and stores it with `to`
    CUtensorMap to;   // output [B,H,Nq,dv_out] 16-bit, 64-column x 128-row boxes (tma_out only)
    int round_dtype;  // dtype the reference's result has before its cast back
    float scale_log2; // softmax scale * log2(e)
    int causal;
    MaskView mask;
    HeadSelect sel;
    const float* q_scale;  // e4m3, and FP32 heads with scaled q/k: [B,H,nt_q] (else nullptr)
    const float* k_scale;  // e4m3, and FP32 heads with scaled q/k: [B,H,nt_k] (else nullptr)
    const float* v_scale;  // e4m3 and FP32 heads: [B,H]
    int64_t nt_q, nt_k;
    int* work_counter;  // zeroed work-item counter (dynamic scheduling), or nullptr (static striding)
    int head_group;     // heads per scheduling group (>= 1): items are handed out group by group,
                        // heaviest query-tile pair first across the group's heads
    unsigned int* status;
    uint64_t timeout_ns;
};
int launch_fmha_tc(const TcLaunch& L, cudaStream_t stream);

// --- fp32 SIMT FMHA ----------------------------------------------------------
struct SimtLaunch {
    const void* q;   // [B,H,Nq,dqk] (q or q_low)
    const void* k;
    const void* v;   // [B,H,Nk,dv]
    int q_dtype, k_dtype, v_dtype;
    int64_t qs[4], ks[4], vs[4];
    int64_t B, H, Nq, Nk;
    int dqk, dv;
    void* out;
    int out_dtype;
    int64_t os[4];
    float scale;
    int causal;
    MaskView mask;
    HeadSelect sel;
};
int launch_fmha_simt(const SimtLaunch& L, cudaStream_t stream);

// --- dense layers (tcgen05 GEMM with a fused epilogue) --------------------------
struct LinearLaunch {
    CUtensorMap tx;      // x [M, K], 64-column x 128-row boxes, 128-byte swizzle
    CUtensorMap tw;      // W [N, K], 64-column x 128-row boxes (half of a 256-column tile per CTA)
    CUtensorMap ty;      // y [M, N], 64-column x 32-row boxes (stores), when tma_io
    CUtensorMap tr;      // resid [M, N], 64-column x 32-row boxes (loads), when tma_io and resid
    const void* bias;    // [N] or null
    const void* resid;   // [M, N] rows at ld_r, or null
    void* y;             // [M, N] rows at ld_y
    int64_t M, N, K;
    int64_t ld_y, ld_r;  // row strides in elements
    int dtype;           // ADA_BF16 or ADA_F16 (x, W, bias, resid and y alike)
    int act;             // 0: none, 1: GELU (erf form)
    int vec;             // 16-byte aligned rows of y and resid
    int tma_io;          // y (and resid) through per-warp shared-memory tiles and TMA
    int n_fastest;       // tile order: 1 = the N tiles of one x row block run side by side (x read from
                         // HBM once, W kept in L2), 0 = the M tiles of one W block (W read once)
    unsigned int* status;
    uint64_t timeout_ns;
};
int launch_linear_tc(const LinearLaunch& L, cudaStream_t stream);

// --- LayerNorm and running statistics ------------------------------------------
struct NormLaunch {
    const void* x;       // [M, E] rows at ld_x
    const void* weight;  // [E] or null
    const void* bias;    // [E] or null
    void* y;             // [M, E] rows at ld_y
    int64_t M, ld_x, ld_y;
    int E;
    int dtype;           // ADA_BF16 or ADA_F16
    float eps;
};
int launch_layer_norm(const NormLaunch& L, cudaStream_t stream);
int launch_record_stats(const float* summary, int64_t* call_count, void* low_rank_calls, int lr_dtype,
                        void* precision_distribution, int pd_dtype, cudaStream_t stream);

// --- attention backward (fp32 CUDA cores) --------------------------------------
struct BwdLaunch {
    const void* q;     // [B,H,Nq,dqk] (q or q_low)
    const void* k;     // [B,H,Nk,dqk]
    const void* v;     // [B,H,Nk,dv]
    const void* out;   // [B,H,Nq,dv] forward output
    const void* dout;  // [B,H,Nq,dv] gradient of the output
    int q_dtype, k_dtype, v_dtype, out_dtype, dout_dtype;
    int64_t qs[4], ks[4], vs[4], os[4], gs[4];
    int64_t B, H, Nq, Nk;
    int dqk, dv;
    float scale;
    int causal;
    MaskView mask;
    HeadSelect sel;
    float* lse;     // [B*H*Nq] workspace
    float* delta;   // [B*H*Nq] workspace
    float* dq;      // [B*H][Nq][dqk], zeroed by the caller (atomic accumulation)
    float* dk;      // [B*H][Nk][dqk]
    float* dv_out;  // [B*H][Nk][dv]
};
int launch_attn_bwd(const BwdLaunch& L, cudaStream_t stream);

}  // namespace ada
