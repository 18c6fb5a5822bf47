/*
 * adaattn_b200.h -- C ABI of the B200 (sm_100a) AdaAttn attention-forward path.
 *
 * Plain pointers, sizes and POD structs only: no C++ or framework types cross
 * this boundary. Every entry point returns ADA_OK (0) or a negative ADA_ERR_*
 * code; ada_get_last_error() gives the message of the calling thread's last
 * failure. All device work is enqueued on the caller's stream (a cudaStream_t
 * passed as void*; NULL is the legacy default stream) and nothing synchronises
 * unless the entry point says so. Device buffers are owned by the caller; an
 * entry point that needs scratch memory takes a caller-provided workspace
 * whose size comes from the matching *_workspace_bytes query.
 *
 * Reference interfaces replaced (paths inside hkevin01/AdaAttn):
 *   - the pybind11 module `_adaattn_cuda`, src/adaattn/kernels/bindings.cpp:140-189
 *     (flash_attention_forward, adaptive_attention_forward, compute_entropy,
 *     estimate_effective_rank, determine_target_ranks), imported at
 *     src/adaattn/kernels/__init__.py:39-48 and called at :76-79, :148-151;
 *   - AdaAttention's analyzer and adaptive core,
 *     src/adaattn/attention/adaattn.py:228-289 and :462-504, and the flash_attn
 *     branch it takes on CUDA, src/adaattn/attention/adaattn.py:421-445.
 */
#ifndef ADAATTN_B200_H
#define ADAATTN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ADA_ABI_VERSION 1

/* ---- status codes ---------------------------------------------------- */
#define ADA_OK               0
#define ADA_ERR_INVALID     -1  /* null pointer or parameter out of range   */
#define ADA_ERR_SHAPE       -2  /* tensor shapes disagree                    */
#define ADA_ERR_DTYPE       -3  /* unsupported element type                  */
#define ADA_ERR_DEVICE      -4  /* no sm_100 device / pointer not on device  */
#define ADA_ERR_LAYOUT      -5  /* stride or alignment the kernels cannot use */
#define ADA_ERR_LAUNCH      -6  /* kernel launch failed                      */
#define ADA_ERR_TIMEOUT     -7  /* a device-side wait hit its time limit     */
#define ADA_ERR_WORKSPACE   -8  /* workspace missing or too small            */
#define ADA_ERR_UNSUPPORTED -9  /* valid request outside what is built       */
#define ADA_ERR_CUDA       -10  /* CUDA runtime error                        */

/* ---- element types ---------------------------------------------------- */
#define ADA_F32   0
#define ADA_F16   1
#define ADA_BF16  2
#define ADA_E4M3  3
#define ADA_BOOL  4   /* one byte per element, nonzero = keep */
#define ADA_I32   5
#define ADA_I64   6
#define ADA_F64   7   /* statistics buffers only */

/* ---- precision codes: the reference's _precision_distribution order
 *      (src/adaattn/attention/adaattn.py:480-485) plus AUTO, which computes
 *      in fp16 (base.py:107) and is counted in the FP32 slot (.get(p, 0)). */
#define ADA_PREC_FP32 0
#define ADA_PREC_FP16 1
#define ADA_PREC_BF16 2
#define ADA_PREC_FP8  3
#define ADA_PREC_AUTO 4

/* A strided view of up to 4 dimensions; strides are in elements. For the
 * attention entry points q/k/v/out are [B, H, N, D] (any strides with the
 * last one equal to 1; a [B, N, H, D] buffer is passed by permuting strides).
 * A mask is [B, H, Nq, Nk] with stride 0 on broadcast dimensions. */
typedef struct AdaTensor {
    void*   data;
    int32_t dtype;
    int32_t ndim;
    int64_t shape[4];
    int64_t stride[4];
} AdaTensor;

/* Analyzer knobs; defaults in brackets follow adaattn.py:57-79, base.py:203. */
typedef struct AdaAnalyzeParams {
    double  rank_threshold;             /* low rank when ne < this [0.95]; compared in double like the reference's Python floats */
    float   scale;                      /* softmax scale [1/sqrt(D)]           */
    float   eps;                        /* entropy epsilon [1e-6]              */
    int32_t enable_adaptive_rank;       /* [1]                                  */
    int32_t enable_adaptive_precision;  /* [1]                                  */
    int32_t default_precision;          /* ADA_PREC_* [FP16]                    */
    int32_t allow_fp8;                  /* [0]                                  */
    int32_t granularity;                /* 0: one decision per (b,h); 1: one per call (reference) */
    int32_t sample_stride;              /* 1: first 64 rows (reference); s>1: rows 0, s, 2s, ... */
    int32_t reserved[2];
} AdaAnalyzeParams;

/* Outputs of ada_analyze (device buffers):
 *   decisions  int32 [B*H*2]  {precision code, low_rank flag} per (b,h)
 *   head_stats f32   [B*H*4]  {normalized entropy, max|score|, max prob, effective rank}
 *   summary    f32   [ADA_SUMMARY_LEN]  see ADA_SUM_* */
#define ADA_SUMMARY_LEN 12
#define ADA_SUM_NE        0
#define ADA_SUM_MAX_SCORE 1
#define ADA_SUM_MAX_PROB  2
#define ADA_SUM_EFF_RANK  3
#define ADA_SUM_N_LOWRANK 4
#define ADA_SUM_N_FP32    5   /* counts per precision slot: FP32(+AUTO), FP16, BF16, FP8 */
#define ADA_SUM_N_FP16    6
#define ADA_SUM_N_BF16    7
#define ADA_SUM_N_FP8     8
#define ADA_SUM_N_TOTAL   9

/* Forward knobs. */
typedef struct AdaFwdParams {
    float   scale;          /* softmax scale applied to q.k (both branches use 1/sqrt(D), adaattn.py:144) */
    int32_t causal;         /* top-left aligned: key j hidden from query i when j > i */
    int32_t fp8_mode;       /* 0: FP8 heads use tile-scaled E4M3 tensor cores; 1: fp16 arithmetic like base.py:106 */
    int32_t static_precision; /* used when decisions == NULL */
    int32_t static_low_rank;  /* used when decisions == NULL */
    int32_t reserved[3];
} AdaFwdParams;

int         ada_abi_version(void);
int         ada_get_last_error(char* buf, size_t len);
/* Reads and clears the library's device status word on the current device
 * (synchronises `stream`). Returns ADA_OK or the first ADA_ERR_* a kernel
 * recorded, e.g. ADA_ERR_TIMEOUT from a bounded wait. */
int         ada_poll_device_status(void* stream);

/* Per-head statistics and decisions of the analyzer sample.
 * Replaces AdaAttention._analyze_attention_pattern (adaattn.py:228-289) and
 * the _adaattn_cuda helpers compute_entropy / estimate_effective_rank /
 * determine_target_ranks (bindings.cpp:101-135) on the attention path.
 * No host synchronisation: the decision is written to device memory. */
size_t      ada_analyze_workspace_bytes(int64_t batch, int64_t heads);
int         ada_analyze(const AdaTensor* q, const AdaTensor* k,
                        const AdaAnalyzeParams* params,
                        int32_t* decisions, float* head_stats, float* summary,
                        void* workspace, size_t workspace_bytes, void* stream);

/* ada_analyze for callers that cannot call cudaMalloc (this entry point has no
 * counterpart in the reference). Same inputs and outputs as ada_analyze, but
 * the per-head scratch lives in a fixed device array inside the library
 * instead of a caller workspace, so the call allocates nothing. Limit:
 * batch * heads <= 65536 (the array is 256 KB and every device that loads the
 * library holds it until the process exits); larger inputs return
 * ADA_ERR_UNSUPPORTED. All calls share the array: calls that overlap on the
 * GPU (other streams, other host threads on the same device) race on it and
 * must be ordered by the caller. The first call on a device resolves the
 * array's address on that device; make it before any stream capture. */
int         ada_analyze_noalloc(const AdaTensor* q, const AdaTensor* k,
                                const AdaAnalyzeParams* params,
                                int32_t* decisions, float* head_stats, float* summary,
                                void* stream);

/* Adaptive attention core on [B,H,N,D]: every (b,h) slice takes the branch
 * (dense / low rank) and the precision its decision names. Replaces
 * AdaAttention._adaptive_attention_forward (adaattn.py:462-504) with
 * _compute_dense_attention (:291-339) and _compute_low_rank_attention
 * (:341-394), and _adaattn_cuda.adaptive_attention_forward (bindings.cpp:73-96).
 *   decisions: device int32 [B*H*2] from ada_analyze, or NULL to use
 *              params->static_precision / static_low_rank for every head.
 *   w_down:    rank_proj_down.weight [r, D] (adaattn.py:133), or NULL when no
 *              head can take the low-rank branch.
 *   mask:      optional [B,H,Nq,Nk] view (bool keeps True; float is added),
 *              as adaattn.py:320-329.
 *   out:       [B,H,Nq,Dv] in the inputs' dtype. */
size_t      ada_attn_fwd_workspace_bytes(const AdaTensor* q, const AdaTensor* k,
                                         const AdaTensor* v, const AdaTensor* w_down,
                                         const int32_t* decisions,
                                         const AdaFwdParams* params,
                                         int32_t possible_precisions_mask,
                                         int32_t low_rank_possible);
int         ada_attn_fwd(const AdaTensor* q, const AdaTensor* k, const AdaTensor* v,
                         const AdaTensor* w_down, const AdaTensor* mask,
                         const int32_t* decisions, const AdaFwdParams* params,
                         int32_t possible_precisions_mask, int32_t low_rank_possible,
                         AdaTensor* out, void* workspace, size_t workspace_bytes,
                         void* stream);

/* ada_attn_fwd for host-resident operands (no counterpart in the reference;
 * the reference's callers pass host tensors and let PyTorch copy them). q, k,
 * v and out point to host memory (pinned for the copies to overlap), each a
 * contiguous [B,H,N,D] tensor. Chunks of consecutive (b, h) slices
 * (chunk_slices per chunk, or about 16 MB of q when 0) stream through
 * `device_buffer` (sized by ada_attn_fwd_host_buffer_bytes): copies in, the
 * forward and copies out run on three internal streams, both PCIe
 * directions overlapping each other and the kernels. Every head takes
 * params->static_precision / static_low_rank (w_down on the device when
 * low rank); no mask. Ordered after prior work on `stream`, which waits for
 * the last copy out: `out` is complete once `stream` is, also when the call
 * fails part-way through. Calls on one device enqueue one at a time on the
 * shared internal streams; a device_buffer must not be shared by calls on
 * different streams (nothing orders one call's first copy into it after the
 * other call's last read of it). */
size_t      ada_attn_fwd_host_buffer_bytes(const AdaTensor* q, const AdaTensor* k,
                                           const AdaTensor* v, const AdaTensor* w_down,
                                           const AdaFwdParams* params, int64_t chunk_slices);
int         ada_attn_fwd_host(const AdaTensor* q, const AdaTensor* k, const AdaTensor* v,
                              const AdaTensor* w_down, const AdaFwdParams* params,
                              AdaTensor* out, int64_t chunk_slices, void* device_buffer,
                              size_t buffer_bytes, void* stream);

/* Gradients of the attention core for autograd (the reference's
 * AdaAttention is differentiable through ATen, tests/unit/
 * test_adaattn_unified.py:146-159): for every selected head, with
 * out = softmax(q k^T * scale + mask) v evaluated in fp32 at the operands'
 * values, writes dq [B,H,Nq,Dqk], dk [B,H,Nk,Dqk] and dv [B,H,Nk,Dv]
 * (contiguous fp32; dq must be zeroed by the caller, it is accumulated).
 * Low-rank heads pass q_low, k_low as q, k (Dqk = r) and chain the
 * projection themselves. decisions: the forward's table, selecting the
 * heads whose low-rank flag equals low_rank (NULL: every head). Uses
 * params->scale and ->causal; mask as in ada_attn_fwd. Dqk, Dv <= 128.
 * Workspace: ada_attn_bwd_workspace_bytes(B, H, Nq) bytes. */
size_t      ada_attn_bwd_workspace_bytes(int64_t batch, int64_t heads, int64_t nq);
int         ada_attn_bwd(const AdaTensor* q, const AdaTensor* k, const AdaTensor* v,
                         const AdaTensor* out, const AdaTensor* dout, const AdaTensor* mask,
                         const int32_t* decisions, int32_t low_rank, const AdaFwdParams* params,
                         AdaTensor* dq, AdaTensor* dk, AdaTensor* dv,
                         void* workspace, size_t workspace_bytes, void* stream);

/* _adaattn_cuda.flash_attention_forward (bindings.cpp:21-68): q, k, v, out are
 * [B, N, H, D] fp16/bf16 (or f32); scale <= 0 means 1/sqrt(D). */
int         ada_flash_attention_forward(const AdaTensor* q, const AdaTensor* k,
                                        const AdaTensor* v, float scale, int32_t causal,
                                        AdaTensor* out, void* stream);

/* _adaattn_cuda.compute_entropy (bindings.cpp:101-109): rows of `weights`
 * (last dimension) -> entropy -sum w*log(w + 1e-10), f32 output with the
 * leading dimensions. estimate_effective_rank (:114-118) is exp(mean of the
 * last entropy dimension); determine_target_ranks (:123-135) maps effective
 * ranks to int64 target ranks. */
int         ada_compute_entropy(const AdaTensor* weights, float* entropy_out, void* stream);
int         ada_estimate_effective_rank(const AdaTensor* weights, float* rank_out, void* stream);
int         ada_determine_target_ranks(const float* effective_rank, int64_t n,
                                       int64_t min_rank, int64_t max_rank, double threshold,
                                       int64_t* ranks_out, void* stream);

/* Randomized truncated SVD of a batch of fp32 matrices, A ~= U diag(S) Vh;
 * replaces adaattn.linalg.low_rank.randomized_svd
 * (src/adaattn/linalg/low_rank.py:56-109) with the Gaussian sketch passed in.
 *   a      [batch, m, n] fp32 (any strides; copied when TMA cannot read it)
 *   omega  [batch, n, k] fp32, k = min(rank + oversampling, min(m, n)) <= 112
 *   n_power power iterations Y = A (A^T Y) (the reference uses 2)
 *   u [batch, m, rank], s [batch, rank] (descending), vh [batch, rank, n] fp32
 * The basis of range(Y) comes from CholeskyQR2 instead of Householder QR; a
 * sketch column that is numerically inside the span of the earlier ones
 * gives a zero basis column. Workspace: 256-byte aligned,
 * ada_rsvd_workspace_bytes() bytes (0 when the arguments are invalid). */
size_t      ada_rsvd_workspace_bytes(const AdaTensor* a, const AdaTensor* omega, int32_t rank);
int         ada_rsvd(const AdaTensor* a, const AdaTensor* omega, int32_t rank, int32_t n_power,
                     AdaTensor* u, AdaTensor* s, AdaTensor* vh,
                     void* workspace, size_t workspace_bytes, void* stream);

/* The module's dense layers on the tensor cores: y = act(x w^T + bias) (+ residual),
 * replacing the nn.Linear calls on either side of the attention path: the
 * q/k/v projections (src/adaattn/attention/adaattn.py:411-418, stacked into
 * one [3E, E] weight for self-attention) and out_proj (:457), plus the
 * host transformer block's feed-forward and residual sums
 * (examples/transformer_integration.py:33-58).
 *   x [M, K], w [N, K] (nn.Linear's weight), y [M, N]: 2-D views, one dtype
 *     (bf16 or fp16), unit column strides; x and w with 16-byte aligned bases
 *     and row strides (so K is a multiple of 8).
 *   bias [N] contiguous or NULL; residual [M, N] or NULL.
 *   activation 0: none, 1: GELU, erf form (nn.GELU()).
 * Rounds like the PyTorch ops it replaces: the Linear's output to the dtype,
 * then the GELU's, then the residual sum's; products accumulate in fp32. */
int         ada_linear(const AdaTensor* x, const AdaTensor* w, const AdaTensor* bias,
                       const AdaTensor* residual, int32_t activation, AdaTensor* y, void* stream);

/* LayerNorm over the last dimension of x [M, E] (bf16 or fp16, unit column
 * stride, 16-byte aligned rows, E a multiple of 8 and <= 2048), weight and
 * bias [E] contiguous in x's dtype (either may be NULL): the host block's
 * nn.LayerNorm (examples/transformer_integration.py:44-45, 81) in fp32
 * arithmetic, rounded once. y [M, E] may alias x. */
int         ada_layer_norm(const AdaTensor* x, const AdaTensor* weight, const AdaTensor* bias,
                           float eps, AdaTensor* y, void* stream);

/* Adds one call's decision summary (ada_analyze's `summary`) to the module's
 * running statistics buffers like adaattn.py:486-498: call_count (int64
 * scalar) += 1, low_rank_calls (scalar) += n_lowrank / total, and
 * precision_distribution[4] += counts / total, each ratio cast to its
 * buffer's dtype (fp32, fp16, bf16 or ADA_F64) and added in that dtype. */
int         ada_record_statistics(const float* summary, AdaTensor* call_count,
                                  AdaTensor* low_rank_calls, AdaTensor* precision_distribution,
                                  void* stream);

/* Test hook for failure detection: launches one block that waits on a device
 * barrier nothing ever signals, bounded by `timeout_ns`; the wait gives up,
 * records ADA_ERR_TIMEOUT in the status word and the kernel returns normally. */
int         ada_debug_bounded_wait(uint64_t timeout_ns, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ADAATTN_B200_H */
