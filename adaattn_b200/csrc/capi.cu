// The C ABI (include/adaattn_b200.h): argument checking, the per-call launch
// plan (which kernels serve which heads, workspace carving, TMA descriptors)
// and the device status word. No entry point here allocates device memory.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "ada_common.cuh"
#include "ada_internal.h"

namespace ada {
namespace {

__device__ unsigned int g_ada_status = 0;

thread_local char g_last_error[512] = {0};

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return code;
}

constexpr int kMaxDevices = 64;
std::mutex g_mu;
unsigned int* g_status_ptr[kMaxDevices] = {nullptr};
int g_cc_major[kMaxDevices] = {0};
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int current_device(int* dev) {
    if (cudaGetDevice(dev) != cudaSuccess) return fail(ADA_ERR_DEVICE, "cudaGetDevice failed");
    if (*dev < 0 || *dev >= kMaxDevices) return fail(ADA_ERR_DEVICE, "device index %d out of range", *dev);
    return ADA_OK;
}

// Per-device setup, done once with that device current: check for sm_100 and
// resolve the device address of the status word.
int device_setup(unsigned int** status) {
    int dev;
    int rc = current_device(&dev);
    if (rc) return rc;
    // Binds the device's primary context to the calling thread (a thread
    // that has only selected the device, e.g. autograd's worker, may have
    // none current, and the driver's tensor-map encoder needs one).
    if (cudaSetDevice(dev) != cudaSuccess) return fail(ADA_ERR_DEVICE, "cudaSetDevice(%d) failed", dev);
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_cc_major[dev] == 0) {
        cudaDeviceProp prop;
        if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess)
            return fail(ADA_ERR_DEVICE, "cudaGetDeviceProperties failed");
        g_cc_major[dev] = prop.major;
    }
    if (g_cc_major[dev] != 10)
        return fail(ADA_ERR_DEVICE, "device %d is sm_%d*, this library is built for sm_100a", dev,
                    g_cc_major[dev]);
    if (g_status_ptr[dev] == nullptr) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_ada_status);
        if (e != cudaSuccess) return fail(ADA_ERR_CUDA, "cudaGetSymbolAddress: %s", cudaGetErrorString(e));
        g_status_ptr[dev] = static_cast<unsigned int*>(p);
    }
    *status = g_status_ptr[dev];
    return ADA_OK;
}

int encoder(PFN_cuTensorMapEncodeTiled_v12000* fn) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_encode == nullptr) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess || p == nullptr)
            return fail(ADA_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
        g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    *fn = g_encode;
    return ADA_OK;
}

uint64_t wait_timeout_ns() {
    static uint64_t v = [] {
        const char* s = getenv("ADA_WAIT_TIMEOUT_MS");
        long ms = s ? atol(s) : 0;
        if (ms <= 0) ms = 4000;
        return static_cast<uint64_t>(ms) * 1000000ull;
    }();
    return v;
}

int elt_bytes(int dtype) {
    switch (dtype) {
        case ADA_F32: return 4;
        case ADA_F16: return 2;
        case ADA_BF16: return 2;
        case ADA_E4M3: return 1;
        case ADA_BOOL: return 1;
        case ADA_I32: return 4;
        case ADA_I64: return 8;
        default: return 0;
    }
}

bool is_float(int dtype) { return dtype == ADA_F32 || dtype == ADA_F16 || dtype == ADA_BF16; }

int check_attn_tensor(const AdaTensor* t, const char* name) {
    if (t == nullptr || t->data == nullptr) return fail(ADA_ERR_INVALID, "%s is null", name);
    if (t->ndim != 4) return fail(ADA_ERR_SHAPE, "%s must be 4-D [B,H,N,D], got %d-D", name, t->ndim);
    if (!is_float(t->dtype)) return fail(ADA_ERR_DTYPE, "%s dtype %d unsupported", name, t->dtype);
    for (int i = 0; i < 4; ++i)
        if (t->shape[i] < 0) return fail(ADA_ERR_SHAPE, "%s has a negative extent", name);
    return ADA_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// TMA-readable in place: innermost stride 1, other strides multiples of 16
// bytes, base 16-byte aligned.
bool tma_ok(const AdaTensor* t) {
    const int eb = elt_bytes(t->dtype);
    if (t->stride[3] != 1 && t->shape[3] > 1) return false;
    if (!aligned16(t->data)) return false;
    for (int i = 0; i < 3; ++i) {
        if (t->shape[i] <= 1) continue;
        if (t->stride[i] <= 0 || ((t->stride[i] * eb) % 16) != 0) return false;
    }
    return true;
}

// 4-D map over [B, H, N, width] (dims innermost first: width, N, H, B) with a
// 128-row x 128-byte box and 128-byte swizzle.
int make_map(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int eb, int64_t width, int64_t n,
             int64_t h, int64_t b, int64_t s_n, int64_t s_h, int64_t s_b) {
    PFN_cuTensorMapEncodeTiled_v12000 enc;
    int rc = encoder(&enc);
    if (rc) return rc;
    auto fix = [&](int64_t s, int64_t ext, int64_t fallback) {
        return (ext <= 1 || s <= 0) ? fallback : s;
    };
    const int64_t rowb = s_n * eb;
    const int64_t fb = ((n * rowb + 15) / 16) * 16;
    cuuint64_t dims[4] = {static_cast<cuuint64_t>(width), static_cast<cuuint64_t>(n > 0 ? n : 1),
                          static_cast<cuuint64_t>(h), static_cast<cuuint64_t>(b)};
    cuuint64_t strides[3] = {static_cast<cuuint64_t>(fix(rowb, n, 128)),
                             static_cast<cuuint64_t>(fix(s_h * eb, h, fb)),
                             static_cast<cuuint64_t>(fix(s_b * eb, b, fb * (h > 0 ? h : 1)))};
    cuuint32_t box[4] = {static_cast<cuuint32_t>(128 / eb), 128, 1, 1};
    cuuint32_t es[4] = {1, 1, 1, 1};
    CUresult r = enc(map, dt, 4, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(ADA_ERR_LAYOUT, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return ADA_OK;
}

// 2-D map over a contiguous row-major [rows, width] 16-bit matrix with a
// box_rows x 128-byte box and 128-byte swizzle (rows past the end read zero).
int make_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int64_t width, int64_t rows,
                int box_rows) {
    PFN_cuTensorMapEncodeTiled_v12000 enc;
    int rc = encoder(&enc);
    if (rc) return rc;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(width), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(width * 2)};
    cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
    cuuint32_t es[2] = {1, 1};
    CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(ADA_ERR_LAYOUT, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return ADA_OK;
}

// 2-D map over a row-major [rows, width] 16-bit matrix whose rows are `ld`
// elements apart, with a box_rows x 128-byte box and 128-byte swizzle.
int make_map_rows(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int64_t width, int64_t rows,
                  int64_t ld, int box_rows) {
    PFN_cuTensorMapEncodeTiled_v12000 enc;
    int rc = encoder(&enc);
    if (rc) return rc;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(width), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>((rows > 1 ? ld : width) * 2)};
    cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
    cuuint32_t es[2] = {1, 1};
    CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(ADA_ERR_LAYOUT, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return ADA_OK;
}

// 3-D map over [batch, rows, width] (innermost first) with a
// box_cols x 128-row box and 128-byte swizzle; strides in elements.
int make_map_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int eb, int64_t width, int64_t rows,
                int64_t batch, int64_t s_row, int64_t s_batch, int box_cols) {
    PFN_cuTensorMapEncodeTiled_v12000 enc;
    int rc = encoder(&enc);
    if (rc) return rc;
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(width), static_cast<cuuint64_t>(rows),
                          static_cast<cuuint64_t>(batch)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(s_row * eb), static_cast<cuuint64_t>(s_batch * eb)};
    cuuint32_t box[3] = {static_cast<cuuint32_t>(box_cols), 128, 1};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = enc(map, dt, 3, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(ADA_ERR_LAYOUT, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return ADA_OK;
}

CUtensorMapDataType tma_dtype(int dtype) {
    switch (dtype) {
        case ADA_F16: return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
        case ADA_BF16: return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
        default: return CU_TENSOR_MAP_DATA_TYPE_UINT8;
    }
}

constexpr uint32_t bit(int p) { return 1u << p; }

// ---------------------------------------------------------------------------
// The forward plan: derived only from shapes, dtypes, flags and the set of
// decisions that can occur, so the workspace query and the call agree.
// ---------------------------------------------------------------------------
struct Plan {
    int in_dtype;
    int64_t B, H, Nq, Nk, D, r;
    uint32_t possible;
    bool low_possible, dense_possible;
    int fp8_mode;
    uint32_t tc16_mask, f16_mask, fp8_mask, fp32_mask;
    bool direct_ok;
    bool v_direct;       // v itself is TMA-readable at the padded width (the kernels read it in place)
    int dqk_dense, dqk_low, dv_pad;
    int64_t ld16_qk, ld16_v;
    bool need16, need32, need8;
    bool split;          // some FP32 heads run on the tensor cores (scaled fp16 operands, split P)
    bool split_low, split_dense;
    bool split_low_direct, split_dense_direct;  // q/k read in place (16-bit region / inputs), not scaled
    bool split_scaled;   // some FP32 heads' q/k are scaled into the split q/k region
    int64_t split_ld;    // row width of the split q/k region
    bool proj_tc_shape;  // low-rank projection can run on the tensor cores
    bool proj_tc;        // ... and will (the weight is 16-byte aligned)
    int64_t nt_q, nt_k;
    size_t off16q, off16k, off16v, off32q, off32k, off8q, off8k, off8v;
    size_t off_amax_q, off_amax_k, off_amax_v, off_sq, off_sk, off_sv;
    size_t offs_q, offs_k, offs_v, offs_sq, offs_sk, offs_sv, offs_amax;
    size_t required;      // bytes the operand regions need
    size_t off_counters;  // work-item counters of the tensor-core launches
    size_t total;         // required + counters
};

constexpr int kMaxCounters = 16;

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

int pad_width(int64_t d) { return d <= 64 ? 64 : 128; }

int build_plan(const AdaTensor* q, const AdaTensor* k, const AdaTensor* v, const AdaTensor* w_down,
               const int32_t* decisions, const AdaFwdParams* p, int32_t possible_mask, int32_t low_possible,
               Plan* P) {
    int rc;
    if ((rc = check_attn_tensor(q, "q")) || (rc = check_attn_tensor(k, "k")) || (rc = check_attn_tensor(v, "v")))
        return rc;
    if (p == nullptr) return fail(ADA_ERR_INVALID, "params is null");
    if (q->dtype != k->dtype || q->dtype != v->dtype)
        return fail(ADA_ERR_DTYPE, "q, k, v must share one dtype");
    if (q->shape[0] != k->shape[0] || q->shape[0] != v->shape[0] || q->shape[1] != k->shape[1] ||
        q->shape[1] != v->shape[1])
        return fail(ADA_ERR_SHAPE, "batch/head extents of q, k, v differ");
    if (k->shape[2] != v->shape[2]) return fail(ADA_ERR_SHAPE, "k and v sequence lengths differ");
    if (q->shape[3] != k->shape[3]) return fail(ADA_ERR_SHAPE, "q and k head dims differ");
    if (v->shape[3] != q->shape[3]) return fail(ADA_ERR_UNSUPPORTED, "value head dim must equal the query head dim");
    std::memset(P, 0, sizeof(*P));
    P->in_dtype = q->dtype;
    P->B = q->shape[0];
    P->H = q->shape[1];
    P->Nq = q->shape[2];
    P->Nk = k->shape[2];
    P->D = q->shape[3];
    if (P->D < 1 || P->D > 128) return fail(ADA_ERR_UNSUPPORTED, "head dim %lld outside [1, 128]", (long long)P->D);
    P->fp8_mode = p->fp8_mode;
    if (decisions == nullptr) {
        if (p->static_precision < 0 || p->static_precision > 4)
            return fail(ADA_ERR_INVALID, "static precision %d", p->static_precision);
        P->possible = bit(p->static_precision);
        P->low_possible = p->static_low_rank != 0;
        P->dense_possible = p->static_low_rank == 0;
    } else {
        P->possible = static_cast<uint32_t>(possible_mask) & 0x1Fu;
        P->low_possible = low_possible != 0;
        P->dense_possible = true;
    }
    if (P->low_possible) {
        if (w_down == nullptr || w_down->data == nullptr)
            return fail(ADA_ERR_INVALID, "low-rank heads need rank_proj_down weights");
        if (w_down->ndim != 2 || w_down->shape[1] != P->D)
            return fail(ADA_ERR_SHAPE, "w_down must be [r, D]");
        if (w_down->stride[1] != 1 || w_down->stride[0] != w_down->shape[1])
            return fail(ADA_ERR_LAYOUT, "w_down must be contiguous");
        if (!is_float(w_down->dtype)) return fail(ADA_ERR_DTYPE, "w_down dtype");
        if (w_down->dtype != P->in_dtype)
            return fail(ADA_ERR_DTYPE, "rank_proj_down dtype must match the inputs' dtype");
        P->r = w_down->shape[0];
        if (P->r < 1 || P->r > 128) return fail(ADA_ERR_UNSUPPORTED, "rank %lld outside [1, 128]", (long long)P->r);
    }
    P->tc16_mask = bit(ADA_PREC_FP16) | bit(ADA_PREC_AUTO) | bit(ADA_PREC_BF16) |
                   (P->fp8_mode == 1 ? bit(ADA_PREC_FP8) : 0u);
    P->f16_mask = bit(ADA_PREC_FP16) | bit(ADA_PREC_AUTO) | (P->fp8_mode == 1 ? bit(ADA_PREC_FP8) : 0u);
    P->fp8_mask = P->fp8_mode == 1 ? 0u : bit(ADA_PREC_FP8);
    P->fp32_mask = bit(ADA_PREC_FP32);
    P->direct_ok = (P->in_dtype == ADA_F16 || P->in_dtype == ADA_BF16) && (P->D == 64 || P->D == 128) &&
                   tma_ok(q) && tma_ok(k) && tma_ok(v);
    P->dqk_dense = pad_width(P->D);
    P->dqk_low = P->low_possible ? pad_width(P->r) : 0;
    // A rank wider than a 64-wide head pads V to 128 as well: the kernels
    // pair a 128-wide Q K^T only with a 128-wide P V.
    P->dv_pad = P->dqk_low > pad_width(P->D) ? P->dqk_low : pad_width(P->D);
    P->v_direct = P->direct_ok && P->dv_pad == P->D;
    P->ld16_qk = P->dqk_dense > P->dqk_low ? P->dqk_dense : P->dqk_low;
    P->ld16_v = P->dv_pad;
    P->need16 = false;
    for (int pc = 0; pc < 5; ++pc) {
        if (!((P->possible >> pc) & 1u) || !((P->tc16_mask >> pc) & 1u)) continue;
        const int cd = ((P->f16_mask >> pc) & 1u) ? ADA_F16 : ADA_BF16;
        if (P->low_possible || cd != P->in_dtype || !P->direct_ok) P->need16 = true;
    }
    P->need32 = ((P->possible & P->fp32_mask) != 0) && P->low_possible;
    P->need8 = (P->possible & P->fp8_mask) != 0;
    P->proj_tc_shape = P->low_possible && P->direct_ok &&
                       ((P->D == 128 && P->r <= 128) || (P->D == 64 && P->r <= 64));
    P->proj_tc = P->proj_tc_shape && (reinterpret_cast<uintptr_t>(w_down->data) & 15u) == 0;
    // FP32 heads of 16-bit inputs (dense, or low rank with r <= 64) run
    // fp32-accurate on the tensor cores (exact 16-bit q/k products, split P);
    // wider ranks and fp32 inputs stay on the CUDA cores. Their q/k are read
    // in place when the tensor-core projection writes q_low/k_low to the
    // 16-bit region (low rank) or the inputs are TMA-readable (dense), else
    // scaled into a region of their own.
    {
        const bool in16 = P->in_dtype == ADA_F16 || P->in_dtype == ADA_BF16;
        const bool fp32 = (P->possible & P->fp32_mask) != 0;
        P->split_low = in16 && fp32 && P->low_possible && P->r <= 64;
        P->split_dense = in16 && fp32 && P->dense_possible;
        P->split_low_direct = P->split_low && P->proj_tc;
        P->split_dense_direct = P->split_dense && P->direct_ok;
        P->split = P->split_low || P->split_dense;
        const bool scaled_low = P->split_low && !P->split_low_direct;
        const bool scaled_dense = P->split_dense && !P->split_dense_direct;
        P->split_scaled = scaled_low || scaled_dense;
        P->split_ld = scaled_dense ? P->dqk_dense : 64;
        if (P->split_low_direct) {
            P->need32 = false;
            P->need16 = true;
        }
    }
    // E4M3 low-rank heads take their projection from the tensor-core kernel,
    // which writes q_low/k_low into the 16-bit region.
    if (P->need8 && P->proj_tc_shape) P->need16 = true;
    P->nt_q = (P->Nq + 127) / 128;
    P->nt_k = (P->Nk + 127) / 128;
    const int64_t BH = P->B * P->H;
    size_t off = 0;
    if (P->need16) {
        P->off16q = off;
        off = align256(off + static_cast<size_t>(BH * P->Nq * P->ld16_qk) * 2);
        P->off16k = off;
        off = align256(off + static_cast<size_t>(BH * P->Nk * P->ld16_qk) * 2);
        P->off16v = off;
        off = align256(off + static_cast<size_t>(BH * P->Nk * P->ld16_v) * 2);
    }
    if (P->need32) {
        P->off32q = off;
        off = align256(off + static_cast<size_t>(BH * P->Nq * P->r) * 4);
        P->off32k = off;
        off = align256(off + static_cast<size_t>(BH * P->Nk * P->r) * 4);
    }
    if (P->split) {
        const int64_t lq = P->split_scaled ? P->split_ld : 0;
        P->offs_q = off;
        off = align256(off + static_cast<size_t>(BH * P->Nq * lq) * 2);
        P->offs_k = off;
        off = align256(off + static_cast<size_t>(BH * P->Nk * lq) * 2);
        P->offs_v = off;
        off = align256(off + static_cast<size_t>(BH * P->Nk * 128) * 2);
        P->offs_sq = off;
        off = align256(off + static_cast<size_t>(BH * P->nt_q) * 4);
        P->offs_sk = off;
        off = align256(off + static_cast<size_t>(BH * P->nt_k) * 4);
        P->offs_sv = off;
        off = align256(off + static_cast<size_t>(BH) * 4);
        P->offs_amax = off;
        off = align256(off + static_cast<size_t>(BH) * 4);
    }
    if (P->need8) {
        P->off8q = off;
        off = align256(off + static_cast<size_t>(BH * P->Nq * 128));
        P->off8k = off;
        off = align256(off + static_cast<size_t>(BH * P->Nk * 128));
        P->off8v = off;
        off = align256(off + static_cast<size_t>(BH * P->Nk * 128));
        P->off_amax_q = off;
        off = align256(off + static_cast<size_t>(BH * P->nt_q) * 4);
        P->off_amax_k = off;
        off = align256(off + static_cast<size_t>(BH * P->nt_k) * 4);
        P->off_amax_v = off;
        off = align256(off + static_cast<size_t>(BH * P->nt_k) * 4);
        P->off_sq = off;
        off = align256(off + static_cast<size_t>(BH * P->nt_q) * 4);
        P->off_sk = off;
        off = align256(off + static_cast<size_t>(BH * P->nt_k) * 4);
        P->off_sv = off;
        off = align256(off + static_cast<size_t>(BH) * 4);
    }
    P->required = off;
    P->off_counters = off;
    P->total = align256(off + kMaxCounters * sizeof(int));
    return ADA_OK;
}

MaskView mask_view(const AdaTensor* m) {
    MaskView mv{};
    if (m == nullptr || m->data == nullptr) return mv;
    mv.data = m->data;
    mv.dtype = m->dtype;
    for (int i = 0; i < 4; ++i) mv.s[i] = m->shape[i] == 1 ? 0 : m->stride[i];
    return mv;
}

int check_mask(const AdaTensor* m, const Plan& P) {
    if (m == nullptr || m->data == nullptr) return ADA_OK;
    if (m->ndim != 4) return fail(ADA_ERR_SHAPE, "mask must be a 4-D [B,H,Nq,Nk] view");
    if (m->dtype != ADA_BOOL && !is_float(m->dtype)) return fail(ADA_ERR_DTYPE, "mask dtype");
    const int64_t want[4] = {P.B, P.H, P.Nq, P.Nk};
    for (int i = 0; i < 4; ++i)
        if (m->shape[i] != want[i] && m->shape[i] != 1)
            return fail(ADA_ERR_SHAPE, "mask extent %d is %lld, expected %lld or 1", i, (long long)m->shape[i],
                        (long long)want[i]);
    return ADA_OK;
}

// Widest vector store (16 or 32 bytes) every output row start allows, or 0.
int out_vec_bytes(const AdaTensor* o) {
    const int eb = elt_bytes(o->dtype);
    if (o->stride[3] != 1) return 0;
    for (int w = 32; w >= 16; w /= 2) {
        bool ok = (reinterpret_cast<uintptr_t>(o->data) % w) == 0;
        for (int i = 0; i < 3; ++i)
            if (((o->stride[i] * eb) % w) != 0) ok = false;
        if (ok) return w;
    }
    return 0;
}

void copy_strides(int64_t* dst, const AdaTensor* t) {
    for (int i = 0; i < 4; ++i) dst[i] = t->stride[i];
}

}  // namespace
}  // namespace ada

namespace ada {
// Lets entry points defined in other files report through ada_get_last_error.
int record_last_error(int code, const char* msg) { return fail(code, "%s", msg); }

int analyze_setup(const AdaTensor* q, const AdaTensor* k, const AdaAnalyzeParams* params, int32_t* decisions,
                  float* head_stats, float* summary, AnalyzeLaunch* L) {
    unsigned int* st;
    int rc = device_setup(&st);
    if (rc) return rc;
    if ((rc = check_attn_tensor(q, "q")) || (rc = check_attn_tensor(k, "k"))) return rc;
    if (params == nullptr || decisions == nullptr || head_stats == nullptr || summary == nullptr)
        return fail(ADA_ERR_INVALID, "null argument");
    if (q->dtype != k->dtype) return fail(ADA_ERR_DTYPE, "q and k dtypes differ");
    if (q->shape[0] != k->shape[0] || q->shape[1] != k->shape[1] || q->shape[3] != k->shape[3])
        return fail(ADA_ERR_SHAPE, "q and k shapes disagree");
    const int64_t B = q->shape[0], H = q->shape[1], Nq = q->shape[2], Nk = k->shape[2], D = q->shape[3];
    if (D < 1 || D > 256) return fail(ADA_ERR_UNSUPPORTED, "analyzer head dim %lld outside [1, 256]", (long long)D);
    if (Nq < 1 || Nk < 1) return fail(ADA_ERR_SHAPE, "empty sequence: the sample size would be 0");
    if (params->default_precision < 0 || params->default_precision > 4)
        return fail(ADA_ERR_INVALID, "default precision %d", params->default_precision);
    const int stride = params->sample_stride > 1 ? params->sample_stride : 1;
    const int64_t n_min = Nq < Nk ? Nq : Nk;
    int64_t S = (n_min + stride - 1) / stride;
    if (S > 64) S = 64;
    *L = AnalyzeLaunch{};
    L->q = q->data;
    L->k = k->data;
    L->dtype = q->dtype;
    L->B = B;
    L->H = H;
    L->Nq = Nq;
    L->Nk = Nk;
    L->D = D;
    copy_strides(L->qs, q);
    copy_strides(L->ks, k);
    L->scale = params->scale;
    L->eps = params->eps;
    L->log_s = std::log(static_cast<double>(S));
    L->S = static_cast<int>(S);
    L->stride = stride;
    L->head_stats = head_stats;
    L->head_sum = nullptr;
    L->decisions = decisions;
    L->summary = summary;
    L->rank_threshold = params->rank_threshold;
    L->enable_rank = params->enable_adaptive_rank;
    L->enable_prec = params->enable_adaptive_precision;
    L->default_prec = params->default_precision;
    L->allow_fp8 = params->allow_fp8;
    L->granularity = params->granularity;
    L->status = st;
    L->timeout_ns = wait_timeout_ns();
    return ADA_OK;
}
int device_status_word(unsigned int** status) { return device_setup(status); }
int tensor_map_encoder(PFN_cuTensorMapEncodeTiled_v12000* fn) { return encoder(fn); }
uint64_t default_wait_timeout_ns() { return wait_timeout_ns(); }
}  // namespace ada

namespace ada {
namespace {
// ---------------------------------------------------------------------------
// Host-resident operands: batch-row chunks streamed through a device staging
// buffer on three streams per device (copy in, forward, copy out), so the
// PCIe transfers in both directions overlap each other and the kernels.
// ---------------------------------------------------------------------------
struct HostPipe {
    std::mutex mu;  // one call's enqueue sequence at a time (the streams and events are shared)
    cudaStream_t s_in = nullptr, s_comp = nullptr, s_out = nullptr;
    cudaEvent_t start = nullptr, in[2] = {nullptr, nullptr}, comp[2] = {nullptr, nullptr},
                out[2] = {nullptr, nullptr};
};
HostPipe g_pipe[kMaxDevices];

int host_pipe(int dev, HostPipe** hp) {
    std::lock_guard<std::mutex> lock(g_mu);
    HostPipe& p = g_pipe[dev];
    if (p.s_in == nullptr) {
        bool ok = cudaStreamCreateWithFlags(&p.s_in, cudaStreamNonBlocking) == cudaSuccess &&
                  cudaStreamCreateWithFlags(&p.s_comp, cudaStreamNonBlocking) == cudaSuccess &&
                  cudaStreamCreateWithFlags(&p.s_out, cudaStreamNonBlocking) == cudaSuccess &&
                  cudaEventCreateWithFlags(&p.start, cudaEventDisableTiming) == cudaSuccess;
        for (int i = 0; ok && i < 2; ++i)
            ok = cudaEventCreateWithFlags(&p.in[i], cudaEventDisableTiming) == cudaSuccess &&
                 cudaEventCreateWithFlags(&p.comp[i], cudaEventDisableTiming) == cudaSuccess &&
                 cudaEventCreateWithFlags(&p.out[i], cudaEventDisableTiming) == cudaSuccess;
        if (!ok) {
            p.s_in = p.s_comp = p.s_out = nullptr;
            return fail(ADA_ERR_CUDA, "creating the host-pipeline streams failed");
        }
    }
    *hp = &p;
    return ADA_OK;
}

// Slice geometry of a host operand: a contiguous [B, H, N, D] tensor, so every
// (b, h) slice is one block and consecutive slices are adjacent; returns the
// bytes per slice, or 0.
int64_t host_slice_bytes(const AdaTensor* t) {
    if (t == nullptr || t->data == nullptr || t->ndim != 4) return 0;
    const int64_t eb = elt_bytes(t->dtype);
    if (eb == 0 || t->stride[3] != 1 || t->stride[2] != t->shape[3]) return 0;
    if (t->shape[1] > 1 && t->stride[1] != t->shape[2] * t->shape[3]) return 0;
    if (t->shape[0] > 1 && t->stride[0] != t->shape[1] * t->shape[2] * t->shape[3]) return 0;
    return t->shape[2] * t->shape[3] * eb;
}

int64_t host_chunk_slices(const AdaTensor* q, int64_t chunk_slices) {
    const int64_t S = q->shape[0] * q->shape[1];
    if (chunk_slices > 0) return chunk_slices < S ? chunk_slices : S;
    // about 16 MB of q per chunk, at least 4 chunks when there are enough slices
    const int64_t sb = host_slice_bytes(q);
    int64_t c = sb > 0 ? (int64_t{16} << 20) / sb : 1;
    const int64_t quarter = (S + 3) / 4;
    if (c > quarter) c = quarter;
    return c < 1 ? 1 : c;
}

// n consecutive slices as one [1, n, N, D] tensor (every slice takes the
// static decision, so which batch row a slice came from does not matter).
AdaTensor chunk_view(const AdaTensor* t, void* base, int64_t n) {
    AdaTensor c = *t;
    c.data = base;
    c.shape[0] = 1;
    c.shape[1] = n;
    c.stride[1] = t->shape[2] * t->shape[3];
    c.stride[0] = n * c.stride[1];
    return c;
}

int host_plan(const AdaTensor* q, const AdaTensor* k, const AdaTensor* v, const AdaTensor* w_down,
              const AdaFwdParams* params, int64_t rows, size_t* ws_bytes, size_t* total) {
    const int64_t rq = host_slice_bytes(q), rk = host_slice_bytes(k), rv = host_slice_bytes(v);
    if (rq == 0 || rk == 0 || rv == 0)
        return fail(ADA_ERR_LAYOUT, "host operands must be contiguous [B,H,N,D] tensors");
    AdaTensor cq = chunk_view(q, q->data, rows), ck = chunk_view(k, k->data, rows), cv = chunk_view(v, v->data, rows);
    Plan P;
    int rc = build_plan(&cq, &ck, &cv, w_down, nullptr, params, 0, params->static_low_rank, &P);
    if (rc) return rc;
    *ws_bytes = P.total;
    // two slots of q, k, v, out (out has q's geometry) + one forward workspace
    const size_t slot = align256(static_cast<size_t>(rq * rows)) * 2 + align256(static_cast<size_t>(rk * rows)) +
                        align256(static_cast<size_t>(rv * rows));
    *total = 2 * slot + align256(P.total);
    return ADA_OK;
}

}  // namespace
}  // namespace ada

using namespace ada;

extern "C" {

int ada_abi_version(void) { return ADA_ABI_VERSION; }

int ada_get_last_error(char* buf, size_t len) {
    if (buf == nullptr || len == 0) return ADA_ERR_INVALID;
    std::strncpy(buf, g_last_error, len - 1);
    buf[len - 1] = '\0';
    return ADA_OK;
}

int ada_poll_device_status(void* stream) {
    unsigned int* st;
    int rc = device_setup(&st);
    if (rc) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    unsigned int word = 0;
    if (cudaMemcpyAsync(&word, st, sizeof(word), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return fail(ADA_ERR_CUDA, "reading the status word failed");
    if (cudaMemsetAsync(st, 0, sizeof(unsigned int), s) != cudaSuccess || cudaStreamSynchronize(s) != cudaSuccess)
        return fail(ADA_ERR_CUDA, "clearing the status word failed");
    if (word == 0) return ADA_OK;
    for (int i = 0; i < 32; ++i)
        if (word & (1u << i)) return fail(-(i + 1), "device reported error code %d", -(i + 1));
    return ADA_OK;
}

size_t ada_analyze_workspace_bytes(int64_t batch, int64_t heads) {
    return align256(static_cast<size_t>(batch > 0 ? batch : 0) * static_cast<size_t>(heads > 0 ? heads : 0) *
                    sizeof(float));
}

int ada_analyze(const AdaTensor* q, const AdaTensor* k, const AdaAnalyzeParams* params, int32_t* decisions,
                float* head_stats, float* summary, void* workspace, size_t workspace_bytes, void* stream) {
    AnalyzeLaunch L{};
    int rc = analyze_setup(q, k, params, decisions, head_stats, summary, &L);
    if (rc) return rc;
    if (L.B * L.H == 0) return ADA_OK;
    if (workspace_bytes < ada_analyze_workspace_bytes(L.B, L.H) || workspace == nullptr)
        return fail(ADA_ERR_WORKSPACE, "analyzer workspace too small");
    L.head_sum = static_cast<float*>(workspace);
    rc = launch_analyze(L, static_cast<cudaStream_t>(stream));
    return rc ? fail(rc, "analyzer launch failed: %s", cudaGetErrorString(cudaGetLastError())) : ADA_OK;
}

size_t ada_attn_fwd_workspace_bytes(const AdaTensor* q, const AdaTensor* k, const AdaTensor* v,
                                    const AdaTensor* w_down, const int32_t* decisions, const AdaFwdParams* params,
                                    int32_t possible_precisions_mask, int32_t low_rank_possible) {
    Plan P;
    if (build_plan(q, k, v, w_down, decisions, params, possible_precisions_mask, low_rank_possible, &P)) return 0;
    return P.total;
}

int ada_attn_fwd(const AdaTensor* q, const AdaTensor* k, const AdaTensor* v, const AdaTensor* w_down,
                 const AdaTensor* mask, const int32_t* decisions, const AdaFwdParams* params,
                 int32_t possible_precisions_mask, int32_t low_rank_possible, AdaTensor* out, void* workspace,
                 size_t workspace_bytes, void* stream) {
    unsigned int* st;
    int rc = device_setup(&st);
    if (rc) return rc;
    Plan P;
    if ((rc = build_plan(q, k, v, w_down, decisions, params, possible_precisions_mask, low_rank_possible, &P)))
        return rc;
    if ((rc = check_attn_tensor(out, "out"))) return rc;
    if (out->dtype != P.in_dtype) return fail(ADA_ERR_DTYPE, "out dtype must match the inputs'");
    if (out->shape[0] != P.B || out->shape[1] != P.H || out->shape[2] != P.Nq || out->shape[3] != P.D)
        return fail(ADA_ERR_SHAPE, "out must be [B,H,Nq,D]");
    if ((rc = check_mask(mask, P))) return rc;
    // Without a workspace the tensor-core launches stride statically over
    // their work items; with one they share dynamically scheduled counters.
    const bool have_ws = workspace != nullptr && workspace_bytes >= P.total;
    if (P.required > 0 && !have_ws)
        return fail(ADA_ERR_WORKSPACE, "workspace needs %zu bytes, got %zu", P.total, workspace_bytes);
    if (P.B * P.H == 0 || P.Nq == 0) return ADA_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (P.Nk == 0) {
        // softmax over no keys, then an empty product: the reference returns zeros.
        return fail(ADA_ERR_SHAPE, "empty key sequence");
    }
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const DecisionSrc dsrc{decisions, params->static_precision, params->static_low_rank};
    const MaskView mv = mask_view(mask);

    // ---- operand preparation -------------------------------------------
    PrepLaunch pl{};
    pl.dec = dsrc;
    pl.q = q->data;
    pl.k = k->data;
    pl.v = v->data;
    pl.in_dtype = P.in_dtype;
    pl.B = P.B;
    pl.H = P.H;
    pl.Nq = P.Nq;
    pl.Nk = P.Nk;
    pl.D = P.D;
    copy_strides(pl.qs, q);
    copy_strides(pl.ks, k);
    copy_strides(pl.vs, v);
    pl.w_down = P.low_possible ? w_down->data : nullptr;
    pl.w_dtype = P.low_possible ? w_down->dtype : ADA_F32;
    pl.r = P.r;
    pl.tc16_mask = P.tc16_mask;
    pl.f16_mask = P.f16_mask;
    pl.direct_ok = P.direct_ok ? 1 : 0;
    pl.mixed16 = (P.direct_ok && P.in_dtype == ADA_BF16) ? 1 : 0;
    pl.v_direct = P.v_direct ? 1 : 0;
    pl.ld16_qk = P.ld16_qk;
    pl.ld16_v = P.ld16_v;
    pl.dqk_dense = P.dqk_dense;
    pl.dqk_low = P.dqk_low;
    pl.dv_pad = P.dv_pad;
    pl.fp32_mask = P.fp32_mask;
    pl.fp8_mask = P.fp8_mask;
    pl.nt_q = P.nt_q;
    pl.nt_k = P.nt_k;
    pl.status = st;
    pl.timeout_ns = wait_timeout_ns();
    // Low-rank q/k projection on the tensor cores when the inputs are 16-bit
    // and TMA-readable; the SIMT projection kernels cover every other case.
    const int r_pad = P.low_possible ? pad_width(P.r) : 0;
    const bool proj_tc = P.proj_tc && (P.need16 || P.need32);
    if (P.need16) {
        pl.ws16_q = ws + P.off16q;
        pl.ws16_k = ws + P.off16k;
        pl.ws16_v = ws + P.off16v;
        // bf16 inputs read in place: q/k of dense heads directly (FP16 heads
        // too), q_low/k_low from the tensor-core projection, v directly or
        // converted to fp16 inside the attention kernel -- nothing to cast.
        const bool nothing_to_cast = P.in_dtype == ADA_BF16 && P.v_direct && (proj_tc || !P.low_possible);
        if (nothing_to_cast) {
        } else if (proj_tc || !P.low_possible) {
            if ((rc = launch_cast16(pl, proj_tc ? 1 : 0, s))) return fail(rc, "operand cast launch failed");
        } else if ((rc = launch_prep16(pl, s))) {
            return fail(rc, "prep16 launch failed");
        }
    }
    if (P.need32) {
        pl.ws32_q = reinterpret_cast<float*>(ws + P.off32q);
        pl.ws32_k = reinterpret_cast<float*>(ws + P.off32k);
        if (!proj_tc && (rc = launch_prep32(pl, s))) return fail(rc, "prep32 launch failed");
    }
    if (proj_tc) {
        ProjLaunch pj;
        std::memset(&pj, 0, sizeof(pj));
        const CUtensorMapDataType dt = tma_dtype(P.in_dtype);
        if ((rc = make_map(&pj.tq, q->data, dt, 2, P.D, P.Nq, P.H, P.B, q->stride[2], q->stride[1], q->stride[0])) ||
            (rc = make_map(&pj.tk, k->data, dt, 2, P.D, P.Nk, P.H, P.B, k->stride[2], k->stride[1], k->stride[0])) ||
            (rc = make_map_2d(&pj.tw, w_down->data, dt, P.D, P.r, r_pad)))
            return rc;
        pj.dec = dsrc;
        pj.in_dtype = P.in_dtype;
        pj.B = P.B;
        pj.H = P.H;
        pj.Nq = P.Nq;
        pj.Nk = P.Nk;
        pj.D = static_cast<int>(P.D);
        pj.r = static_cast<int>(P.r);
        pj.r_pad = r_pad;
        // Only precisions whose operand region exists are written.
        pj.tc16_mask = P.need16 ? (P.tc16_mask & P.possible) : 0u;
        pj.in16_mask = (P.need8 ? (P.fp8_mask & P.possible) : 0u) |
                       (P.split_low_direct ? (P.fp32_mask & P.possible) : 0u);
        pj.f16_mask = P.f16_mask;
        pj.fp32_mask = P.need32 ? (P.fp32_mask & P.possible) : 0u;
        pj.ws16_q = pl.ws16_q;
        pj.ws16_k = pl.ws16_k;
        pj.ld16 = P.ld16_qk;
        pj.ws32_q = pl.ws32_q;
        pj.ws32_k = pl.ws32_k;
        pj.status = st;
        pj.timeout_ns = wait_timeout_ns();
        // Outputs through TMA stores when the rank pads to 64 columns.
        if (r_pad == 64 && P.Nq > 0 && P.Nk > 0) {
            const int64_t BH = P.B * P.H;
            if ((pj.tc16_mask | pj.in16_mask) != 0u) {
                const int64_t l = P.ld16_qk;
                if ((rc = make_map_3d(&pj.to16_q, pj.ws16_q, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, l, P.Nq, BH, l,
                                      P.Nq * l, 64)) ||
                    (rc = make_map_3d(&pj.to16_k, pj.ws16_k, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, l, P.Nk, BH, l,
                                      P.Nk * l, 64)))
                    return rc;
                pj.tma16 = 1;
            }
            if (pj.fp32_mask != 0u && (P.r % 4) == 0) {
                if ((rc = make_map_3d(&pj.to32_q, pj.ws32_q, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, P.r, P.Nq, BH, P.r,
                                      P.Nq * P.r, 32)) ||
                    (rc = make_map_3d(&pj.to32_k, pj.ws32_k, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, P.r, P.Nk, BH, P.r,
                                      P.Nk * P.r, 32)))
                    return rc;
                pj.tma32 = 1;
            }
        }
        if ((rc = launch_proj_tc(pj, s))) return fail(rc, "tensor-core projection launch failed");
    }
    if (P.need8) {
        pl.ws8_q = ws + P.off8q;
        pl.ws8_k = ws + P.off8k;
        pl.ws8_v = ws + P.off8v;
        pl.amax_q = reinterpret_cast<float*>(ws + P.off_amax_q);
        pl.amax_k = reinterpret_cast<float*>(ws + P.off_amax_k);
        pl.amax_v = reinterpret_cast<float*>(ws + P.off_amax_v);
        pl.scale_q = reinterpret_cast<float*>(ws + P.off_sq);
        pl.scale_k = reinterpret_cast<float*>(ws + P.off_sk);
        pl.scale_v = reinterpret_cast<float*>(ws + P.off_sv);
        pl.low_src16 = proj_tc ? 1 : 0;
        if ((rc = launch_prep8(pl, s))) return fail(rc, "prep8 launch failed");
    }

    if (P.split) {
        pl.split_mask = P.fp32_mask;
        pl.split_low = P.split_low ? 1 : 0;
        pl.split_dense = P.split_dense ? 1 : 0;
        pl.split_qk_low = (P.split_low && !P.split_low_direct) ? 1 : 0;
        pl.split_qk_dense = (P.split_dense && !P.split_dense_direct) ? 1 : 0;
        pl.split_ld = P.split_ld;
        pl.wss_q = reinterpret_cast<uint16_t*>(ws + P.offs_q);
        pl.wss_k = reinterpret_cast<uint16_t*>(ws + P.offs_k);
        pl.wss_v = reinterpret_cast<uint16_t*>(ws + P.offs_v);
        pl.split_sq = reinterpret_cast<float*>(ws + P.offs_sq);
        pl.split_sk = reinterpret_cast<float*>(ws + P.offs_sk);
        pl.split_sv = reinterpret_cast<float*>(ws + P.offs_sv);
        pl.split_amax_v = reinterpret_cast<unsigned int*>(ws + P.offs_amax);
        if (cudaMemsetAsync(pl.split_amax_v, 0, static_cast<size_t>(P.B * P.H) * 4, s) != cudaSuccess)
            return fail(ADA_ERR_CUDA, "clearing the split amax failed");
        if ((rc = launch_split(pl, s))) return fail(rc, "split operand launch failed");
    }

    // ---- tensor-core launches ---------------------------------------------
    const float log2e = 1.4426950408889634f;
    int* counters = have_ws ? reinterpret_cast<int*>(ws + P.off_counters) : nullptr;
    int next_counter = 0;
    if (counters != nullptr && cudaMemsetAsync(counters, 0, kMaxCounters * sizeof(int), s) != cudaSuccess)
        return fail(ADA_ERR_CUDA, "clearing the work counters failed");
    // Item order. A job of fewer than 8 work items per SM (a shard of a few
    // dozen heads) takes its items in head groups, heaviest query-tile pair
    // first across each group: measured on B1 H32 N4096 causal, 667-704 ->
    // 827-910 TFLOP/s (B2 H32: 784-830 -> 872-935), as the CTAs that take the
    // last items get light ones. Larger jobs keep the head-major order (group
    // of 1), whose K/V reuse in L2 is tighter (B8 H32 in the grouped order:
    // 966 against 997 TFLOP/s). Heads per group:
    // as many as keep their K and V (16-bit, up to 128 columns each) within
    // ~48 MB of L2, at most 16.
    int sms = 0;
    {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) !=
                                                       cudaSuccess || sms <= 0)
            sms = 148;
    }
    const int64_t kv_head_bytes = (P.Nk > 0 ? P.Nk : 1) * 2 * 128 * 2;
    const int64_t work_items = P.B * P.H * ((P.Nq + 255) / 256);
    const int64_t head_group =
        work_items < 8 * static_cast<int64_t>(sms)  // (so the kernel's grouped order fits 32-bit indices)
            ? std::max<int64_t>(1, std::min<int64_t>(16, (int64_t(48) << 20) / kv_head_bytes))
            : 1;
    auto base_tc = [&](TcLaunch& L) {
        std::memset(&L, 0, sizeof(L));
        L.head_group = static_cast<int>(head_group);
        L.B = P.B;
        L.H = P.H;
        L.Nq = P.Nq;
        L.Nk = P.Nk;
        L.dv_out = static_cast<int>(P.D);
        L.out = out->data;
        L.out_dtype = out->dtype;
        copy_strides(L.os, out);
        L.out_vec = out_vec_bytes(out);
        L.scale_log2 = params->scale * log2e;
        L.causal = params->causal;
        L.mask = mv;
        L.status = st;
        L.timeout_ns = wait_timeout_ns();
        L.nt_q = P.nt_q;
        L.nt_k = P.nt_k;
        L.work_counter = (counters != nullptr && next_counter < kMaxCounters) ? counters + next_counter++ : nullptr;
    };
    for (int cdi = 0; cdi < 2; ++cdi) {
        const int cd = cdi == 0 ? ADA_F16 : ADA_BF16;
        const uint32_t pm = P.possible & P.tc16_mask & (cd == ADA_F16 ? P.f16_mask : ~P.f16_mask);
        if (pm == 0) continue;
        const CUtensorMapDataType dt = tma_dtype(cd);
        for (int low = 0; low < 2; ++low) {
            if (low ? !P.low_possible : !P.dense_possible) continue;
            TcLaunch L;
            base_tc(L);
            L.elt = cd == ADA_BF16 ? 1 : 0;
            L.round_dtype = cd;
            L.sel = HeadSelect{decisions, pm, low};
            const bool direct = !low && cd == P.in_dtype && P.direct_ok;
            // FP16 heads of bf16 inputs: bf16 q, k in place, v from the cast region
            const bool mixed = !low && cd == ADA_F16 && P.in_dtype == ADA_BF16 && P.direct_ok;
            // v of 16-bit heads read in place (bf16 v of FP16 heads converted in the kernel)
            const bool v_in_place = P.v_direct && (cd == P.in_dtype || (cd == ADA_F16 && P.in_dtype == ADA_BF16));
            if (mixed) {
                L.elt = 5;
                L.dqk = static_cast<int>(P.D);
                L.dv = P.dv_pad;
                const CUtensorMapDataType bf = tma_dtype(ADA_BF16);
                const int64_t lv = P.ld16_v;
                if ((rc = make_map(&L.tq, q->data, bf, 2, P.D, P.Nq, P.H, P.B, q->stride[2], q->stride[1], q->stride[0])) ||
                    (rc = make_map(&L.tk, k->data, bf, 2, P.D, P.Nk, P.H, P.B, k->stride[2], k->stride[1], k->stride[0])))
                    return rc;
                if (v_in_place) {
                    L.v_convert = 1;
                    rc = make_map(&L.tv, v->data, bf, 2, P.D, P.Nk, P.H, P.B, v->stride[2], v->stride[1], v->stride[0]);
                } else {
                    rc = make_map(&L.tv, ws + P.off16v, dt, 2, L.dv, P.Nk, P.H, P.B, lv, P.Nk * lv, P.H * P.Nk * lv);
                }
                if (rc) return rc;
            } else if (direct) {
                L.dqk = static_cast<int>(P.D);
                L.dv = static_cast<int>(P.D);
                if ((rc = make_map(&L.tq, q->data, dt, 2, P.D, P.Nq, P.H, P.B, q->stride[2], q->stride[1], q->stride[0])) ||
                    (rc = make_map(&L.tk, k->data, dt, 2, P.D, P.Nk, P.H, P.B, k->stride[2], k->stride[1], k->stride[0])) ||
                    (rc = make_map(&L.tv, v->data, dt, 2, P.D, P.Nk, P.H, P.B, v->stride[2], v->stride[1], v->stride[0])))
                    return rc;
            } else {
                L.dqk = low ? P.dqk_low : P.dqk_dense;
                L.dv = P.dv_pad;
                const int64_t l = P.ld16_qk, lv = P.ld16_v;
                if ((rc = make_map(&L.tq, ws + P.off16q, dt, 2, L.dqk, P.Nq, P.H, P.B, l, P.Nq * l, P.H * P.Nq * l)) ||
                    (rc = make_map(&L.tk, ws + P.off16k, dt, 2, L.dqk, P.Nk, P.H, P.B, l, P.Nk * l, P.H * P.Nk * l)))
                    return rc;
                if (v_in_place) {
                    L.v_convert = cd != P.in_dtype ? 1 : 0;
                    rc = make_map(&L.tv, v->data, tma_dtype(P.in_dtype), 2, P.D, P.Nk, P.H, P.B, v->stride[2],
                                  v->stride[1], v->stride[0]);
                } else {
                    rc = make_map(&L.tv, ws + P.off16v, dt, 2, L.dv, P.Nk, P.H, P.B, lv, P.Nk * lv, P.H * P.Nk * lv);
                }
                if (rc) return rc;
            }
            // 16-bit output through TMA stores when every row start is
            // 16-byte aligned (the epilogue stages the tile in shared memory).
            if (L.dqk == 128 && L.dv == 128 && (out->dtype == ADA_F16 || out->dtype == ADA_BF16) && out->stride[3] == 1 &&
                out_vec_bytes(out) >= 16 && P.Nq > 0) {
                if ((rc = make_map(&L.to, out->data, tma_dtype(out->dtype), 2, P.D, P.Nq, P.H, P.B, out->stride[2],
                                   out->stride[1], out->stride[0])))
                    return rc;
                L.tma_out = 1;
            }
            if ((rc = launch_fmha_tc(L, s))) return fail(rc, "tensor-core attention launch failed (%d,%d)", L.dqk, L.dv);
        }
    }
    if (P.need8) {
        for (int low = 0; low < 2; ++low) {
            if (low ? !P.low_possible : !P.dense_possible) continue;
            TcLaunch L;
            base_tc(L);
            L.elt = 2;
            L.round_dtype = ADA_F16;  // the reference's FP8 mode yields fp16 results
            L.sel = HeadSelect{decisions, P.fp8_mask, low};
            L.dqk = 128;
            L.dv = 128;
            L.q_scale = reinterpret_cast<float*>(ws + P.off_sq);
            L.k_scale = reinterpret_cast<float*>(ws + P.off_sk);
            L.v_scale = reinterpret_cast<float*>(ws + P.off_sv);
            const CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_UINT8;
            if ((rc = make_map(&L.tq, ws + P.off8q, dt, 1, 128, P.Nq, P.H, P.B, 128, P.Nq * 128, P.H * P.Nq * 128)) ||
                (rc = make_map(&L.tk, ws + P.off8k, dt, 1, 128, P.Nk, P.H, P.B, 128, P.Nk * 128, P.H * P.Nk * 128)) ||
                (rc = make_map(&L.tv, ws + P.off8v, dt, 1, 128, P.Nk, P.H, P.B, 128, P.Nk * 128, P.H * P.Nk * 128)))
                return rc;
            if ((rc = launch_fmha_tc(L, s))) return fail(rc, "E4M3 attention launch failed");
        }
    }
    for (int low = 0; low < 2; ++low) {
        if (!(low ? P.split_low : P.split_dense)) continue;
        TcLaunch L;
        base_tc(L);
        const bool direct = low ? P.split_low_direct : P.split_dense_direct;
        L.elt = (direct && P.in_dtype == ADA_BF16) ? 4 : 3;
        L.round_dtype = ADA_F32;
        L.sel = HeadSelect{decisions, P.fp32_mask, low};
        L.dv = 128;
        L.v_scale = reinterpret_cast<float*>(ws + P.offs_sv);
        const CUtensorMapDataType f16 = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
        if (direct && low) {
            // q_low/k_low in the 16-bit region, inputs' dtype, 64 columns
            L.dqk = 64;
            const CUtensorMapDataType dt = tma_dtype(P.in_dtype);
            const int64_t l = P.ld16_qk;
            if ((rc = make_map(&L.tq, ws + P.off16q, dt, 2, 64, P.Nq, P.H, P.B, l, P.Nq * l, P.H * P.Nq * l)) ||
                (rc = make_map(&L.tk, ws + P.off16k, dt, 2, 64, P.Nk, P.H, P.B, l, P.Nk * l, P.H * P.Nk * l)))
                return rc;
        } else if (direct) {
            L.dqk = static_cast<int>(P.D);
            const CUtensorMapDataType dt = tma_dtype(P.in_dtype);
            if ((rc = make_map(&L.tq, q->data, dt, 2, P.D, P.Nq, P.H, P.B, q->stride[2], q->stride[1], q->stride[0])) ||
                (rc = make_map(&L.tk, k->data, dt, 2, P.D, P.Nk, P.H, P.B, k->stride[2], k->stride[1], k->stride[0])))
                return rc;
        } else {
            L.dqk = low ? 64 : P.dqk_dense;
            L.q_scale = reinterpret_cast<float*>(ws + P.offs_sq);
            L.k_scale = reinterpret_cast<float*>(ws + P.offs_sk);
            const int64_t l = P.split_ld;
            if ((rc = make_map(&L.tq, ws + P.offs_q, f16, 2, L.dqk, P.Nq, P.H, P.B, l, P.Nq * l, P.H * P.Nq * l)) ||
                (rc = make_map(&L.tk, ws + P.offs_k, f16, 2, L.dqk, P.Nk, P.H, P.B, l, P.Nk * l, P.H * P.Nk * l)))
                return rc;
        }
        if ((rc = make_map(&L.tv, ws + P.offs_v, f16, 2, 128, P.Nk, P.H, P.B, 128, P.Nk * 128, P.H * P.Nk * 128)))
            return rc;
        if (L.dqk == 128 && P.D == 128 && (out->dtype == ADA_F16 || out->dtype == ADA_BF16) && out->stride[3] == 1 &&
            out_vec_bytes(out) >= 16) {
            if ((rc = make_map(&L.to, out->data, tma_dtype(out->dtype), 2, P.D, P.Nq, P.H, P.B, out->stride[2],
                               out->stride[1], out->stride[0])))
                return rc;
            L.tma_out = 1;
        }
        if ((rc = launch_fmha_tc(L, s))) return fail(rc, "fp32 tensor-core attention launch failed");
    }
    // ---- remaining FP32 heads (fp32 inputs, ranks above 64) on the CUDA cores ----
    if (P.possible & P.fp32_mask) {
        for (int low = 0; low < 2; ++low) {
            if (low ? (!P.low_possible || P.split_low) : (!P.dense_possible || P.split_dense)) continue;
            SimtLaunch L{};
            L.B = P.B;
            L.H = P.H;
            L.Nq = P.Nq;
            L.Nk = P.Nk;
            L.v = v->data;
            L.v_dtype = P.in_dtype;
            copy_strides(L.vs, v);
            L.dv = static_cast<int>(P.D);
            L.out = out->data;
            L.out_dtype = out->dtype;
            copy_strides(L.os, out);
            L.scale = params->scale;
            L.causal = params->causal;
            L.mask = mv;
            L.sel = HeadSelect{decisions, P.fp32_mask, low};
            if (low) {
                L.q = ws + P.off32q;
                L.k = ws + P.off32k;
                L.q_dtype = L.k_dtype = ADA_F32;
                const int64_t r = P.r;
                const int64_t qs[4] = {P.H * P.Nq * r, P.Nq * r, r, 1};
                const int64_t ks[4] = {P.H * P.Nk * r, P.Nk * r, r, 1};
                std::memcpy(L.qs, qs, sizeof(qs));
                std::memcpy(L.ks, ks, sizeof(ks));
                L.dqk = static_cast<int>(r);
            } else {
                L.q = q->data;
                L.k = k->data;
                L.q_dtype = L.k_dtype = P.in_dtype;
                copy_strides(L.qs, q);
                copy_strides(L.ks, k);
                L.dqk = static_cast<int>(P.D);
            }
            if ((rc = launch_fmha_simt(L, s))) return fail(rc, "fp32 attention launch failed");
        }
    }
    return ADA_OK;
}

int ada_flash_attention_forward(const AdaTensor* q, const AdaTensor* k, const AdaTensor* v, float scale,
                                int32_t causal, AdaTensor* out, void* stream) {
    // [B, N, H, D] views -> [B, H, N, D] by swapping the middle extents.
    auto perm = [](const AdaTensor* t) {
        AdaTensor r = *t;
        if (t->ndim == 4) {
            r.shape[1] = t->shape[2];
            r.shape[2] = t->shape[1];
            r.stride[1] = t->stride[2];
            r.stride[2] = t->stride[1];
        }
        return r;
    };
    int rc;
    if ((rc = check_attn_tensor(q, "q")) || (rc = check_attn_tensor(out, "out"))) return rc;
    AdaTensor qp = perm(q), kp = perm(k), vp = perm(v), op = perm(out);
    AdaFwdParams p{};
    p.scale = scale > 0.f ? scale : 1.f / std::sqrt(static_cast<float>(q->shape[3]));
    p.causal = causal;
    p.static_precision = q->dtype == ADA_F16 ? ADA_PREC_FP16 : (q->dtype == ADA_BF16 ? ADA_PREC_BF16 : ADA_PREC_FP32);
    p.static_low_rank = 0;
    return ada_attn_fwd(&qp, &kp, &vp, nullptr, nullptr, nullptr, &p, 0, 0, &op, nullptr, 0, stream);
}

int ada_compute_entropy(const AdaTensor* w, float* entropy_out, void* stream) {
    unsigned int* st;
    int rc = device_setup(&st);
    if (rc) return rc;
    if (w == nullptr || w->data == nullptr || entropy_out == nullptr) return fail(ADA_ERR_INVALID, "null argument");
    if (w->ndim < 1 || w->ndim > 4 || !is_float(w->dtype)) return fail(ADA_ERR_SHAPE, "weights must be 1-4-D float");
    int64_t expect = 1, rows = 1;
    for (int i = w->ndim - 1; i >= 0; --i) {
        if (w->stride[i] != expect && w->shape[i] > 1) return fail(ADA_ERR_LAYOUT, "weights must be contiguous");
        expect *= w->shape[i];
        if (i < w->ndim - 1) rows *= w->shape[i];
    }
    rc = launch_entropy_rows(w->data, w->dtype, rows, w->shape[w->ndim - 1], entropy_out,
                             static_cast<cudaStream_t>(stream));
    return rc ? fail(rc, "entropy launch failed") : ADA_OK;
}

int ada_estimate_effective_rank(const AdaTensor* w, float* rank_out, void* stream) {
    unsigned int* st;
    int rc = device_setup(&st);
    if (rc) return rc;
    if (w == nullptr || w->data == nullptr || rank_out == nullptr) return fail(ADA_ERR_INVALID, "null argument");
    if (w->ndim < 2 || w->ndim > 4 || !is_float(w->dtype)) return fail(ADA_ERR_SHAPE, "weights must be 2-4-D float");
    int64_t expect = 1, groups = 1;
    for (int i = w->ndim - 1; i >= 0; --i) {
        if (w->stride[i] != expect && w->shape[i] > 1) return fail(ADA_ERR_LAYOUT, "weights must be contiguous");
        expect *= w->shape[i];
        if (i < w->ndim - 2) groups *= w->shape[i];
    }
    rc = launch_effective_rank(w->data, w->dtype, groups, w->shape[w->ndim - 2], w->shape[w->ndim - 1], rank_out,
                               static_cast<cudaStream_t>(stream));
    return rc ? fail(rc, "effective-rank launch failed") : ADA_OK;
}

int ada_determine_target_ranks(const float* eff, int64_t n, int64_t min_rank, int64_t max_rank, double threshold,
                               int64_t* ranks_out, void* stream) {
    unsigned int* st;
    int rc = device_setup(&st);
    if (rc) return rc;
    if ((eff == nullptr || ranks_out == nullptr) && n > 0) return fail(ADA_ERR_INVALID, "null argument");
    rc = launch_target_ranks(eff, n, min_rank, max_rank, threshold, ranks_out, static_cast<cudaStream_t>(stream));
    return rc ? fail(rc, "target-rank launch failed") : ADA_OK;
}

size_t ada_attn_fwd_host_buffer_bytes(const AdaTensor* q, const AdaTensor* k, const AdaTensor* v,
                                      const AdaTensor* w_down, const AdaFwdParams* params, int64_t chunk_slices) {
    if (q == nullptr || k == nullptr || v == nullptr || params == nullptr || q->ndim != 4) return 0;
    size_t ws = 0, total = 0;
    if (host_plan(q, k, v, w_down, params, host_chunk_slices(q, chunk_slices), &ws, &total)) return 0;
    return total;
}

int ada_attn_fwd_host(const AdaTensor* q, const AdaTensor* k, const AdaTensor* v, const AdaTensor* w_down,
                      const AdaFwdParams* params, AdaTensor* out, int64_t chunk_slices, void* device_buffer,
                      size_t buffer_bytes, void* stream) {
    unsigned int* st;
    int rc = device_setup(&st);
    if (rc) return rc;
    int dev;
    if ((rc = current_device(&dev))) return rc;
    if (q == nullptr || k == nullptr || v == nullptr || out == nullptr || params == nullptr)
        return fail(ADA_ERR_INVALID, "null argument");
    if (q->ndim != 4 || k->ndim != 4 || v->ndim != 4 || out->ndim != 4)
        return fail(ADA_ERR_SHAPE, "host operands are [B,H,N,D]");
    const int64_t B = q->shape[0] * q->shape[1];  // (b, h) slices
    const AdaTensor* others[3] = {k, v, out};
    for (const AdaTensor* t : others)
        if (t->shape[0] != q->shape[0] || t->shape[1] != q->shape[1])
            return fail(ADA_ERR_SHAPE, "batch or head extents differ");
    const int64_t ro = host_slice_bytes(out);
    if (ro == 0 || ro != host_slice_bytes(q) || out->dtype != q->dtype)
        return fail(ADA_ERR_LAYOUT, "out must be a contiguous host [B,H,Nq,D] buffer shaped like q");
    const int64_t rows = host_chunk_slices(q, chunk_slices);
    size_t ws_bytes = 0, total = 0;
    if ((rc = host_plan(q, k, v, w_down, params, rows, &ws_bytes, &total))) return rc;
    if (device_buffer == nullptr || buffer_bytes < total)
        return fail(ADA_ERR_WORKSPACE, "device buffer needs %zu bytes, got %zu", total, buffer_bytes);
    if (B == 0) return ADA_OK;
    HostPipe* hp;
    if ((rc = host_pipe(dev, &hp))) return rc;
    std::lock_guard<std::mutex> pipe_lock(hp->mu);
    const int64_t rq = host_slice_bytes(q), rk = host_slice_bytes(k), rv = host_slice_bytes(v);
    uint8_t* base = static_cast<uint8_t*>(device_buffer);
    const size_t sq = align256(static_cast<size_t>(rq * rows)), sk = align256(static_cast<size_t>(rk * rows)),
                 sv = align256(static_cast<size_t>(rv * rows));
    const size_t slot = 2 * sq + sk + sv;
    void* ws = base + 2 * slot;
    cudaStream_t caller = static_cast<cudaStream_t>(stream);
    auto ck = [&](cudaError_t e, const char* what) {
        return e == cudaSuccess ? ADA_OK : fail(ADA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    };
    if ((rc = ck(cudaEventRecord(hp->start, caller), "event record")) ||
        (rc = ck(cudaStreamWaitEvent(hp->s_in, hp->start, 0), "stream wait")) ||
        (rc = ck(cudaStreamWaitEvent(hp->s_comp, hp->start, 0), "stream wait")) ||
        (rc = ck(cudaStreamWaitEvent(hp->s_out, hp->start, 0), "stream wait")))
        return rc;
    // After a failure part-way through, work already queued on the internal
    // streams keeps running: the caller's stream waits for all of it, so the
    // caller may reuse device_buffer and the host buffers once `stream` is done.
    auto join_on_error = [&](int code) {
        cudaStream_t internal[3] = {hp->s_in, hp->s_comp, hp->s_out};
        for (cudaStream_t s : internal)
            if (cudaEventRecord(hp->start, s) == cudaSuccess) cudaStreamWaitEvent(caller, hp->start, 0);
        return code;
    };
    const int64_t nchunks = (B + rows - 1) / rows;
    int last = 0;
    for (int64_t c = 0; c < nchunks; ++c) {
        const int sl = static_cast<int>(c & 1);
        const int64_t r0 = c * rows, n = (B - r0) < rows ? (B - r0) : rows;
        uint8_t* dq = base + sl * slot;
        uint8_t* dk = dq + sq;
        uint8_t* dv = dk + sk;
        uint8_t* dout = dv + sv;
        // copy in once the forward two chunks back has read this slot
        if (c >= 2 && (rc = ck(cudaStreamWaitEvent(hp->s_in, hp->comp[sl], 0), "stream wait"))) return join_on_error(rc);
        if ((rc = ck(cudaMemcpyAsync(dq, static_cast<const uint8_t*>(q->data) + r0 * rq, n * rq,
                                     cudaMemcpyHostToDevice, hp->s_in), "copy of q")) ||
            (rc = ck(cudaMemcpyAsync(dk, static_cast<const uint8_t*>(k->data) + r0 * rk, n * rk,
                                     cudaMemcpyHostToDevice, hp->s_in), "copy of k")) ||
            (rc = ck(cudaMemcpyAsync(dv, static_cast<const uint8_t*>(v->data) + r0 * rv, n * rv,
                                     cudaMemcpyHostToDevice, hp->s_in), "copy of v")) ||
            (rc = ck(cudaEventRecord(hp->in[sl], hp->s_in), "event record")))
            return join_on_error(rc);
        // forward once the inputs landed and the copy out two chunks back has read the output slot
        if ((rc = ck(cudaStreamWaitEvent(hp->s_comp, hp->in[sl], 0), "stream wait"))) return join_on_error(rc);
        if (c >= 2 && (rc = ck(cudaStreamWaitEvent(hp->s_comp, hp->out[sl], 0), "stream wait"))) return join_on_error(rc);
        AdaTensor cq = chunk_view(q, dq, n), ckt = chunk_view(k, dk, n), cv = chunk_view(v, dv, n),
                  co = chunk_view(out, dout, n);
        if ((rc = ada_attn_fwd(&cq, &ckt, &cv, w_down, nullptr, nullptr, params, 0, params->static_low_rank, &co,
                               ws, ws_bytes, hp->s_comp)))
            return join_on_error(rc);
        if ((rc = ck(cudaEventRecord(hp->comp[sl], hp->s_comp), "event record"))) return join_on_error(rc);
        // copy out
        if ((rc = ck(cudaStreamWaitEvent(hp->s_out, hp->comp[sl], 0), "stream wait")) ||
            (rc = ck(cudaMemcpyAsync(static_cast<uint8_t*>(out->data) + r0 * ro, dout, n * ro,
                                     cudaMemcpyDeviceToHost, hp->s_out), "copy of out")) ||
            (rc = ck(cudaEventRecord(hp->out[sl], hp->s_out), "event record")))
            return join_on_error(rc);
        last = sl;
    }
    // the caller's stream continues after the last copy out (copies out run in order)
    return ck(cudaStreamWaitEvent(caller, hp->out[last], 0), "stream wait");
}

size_t ada_attn_bwd_workspace_bytes(int64_t batch, int64_t heads, int64_t nq) {
    if (batch < 0 || heads < 0 || nq < 0) return 0;
    return 2 * align256(static_cast<size_t>(batch) * static_cast<size_t>(heads) * static_cast<size_t>(nq) *
                        sizeof(float));
}

int ada_attn_bwd(const AdaTensor* q, const AdaTensor* k, const AdaTensor* v, const AdaTensor* out,
                 const AdaTensor* dout, const AdaTensor* mask, const int32_t* decisions, int32_t low_rank,
                 const AdaFwdParams* params, AdaTensor* dq, AdaTensor* dk, AdaTensor* dv, void* workspace,
                 size_t workspace_bytes, void* stream) {
    unsigned int* st;
    int rc = device_setup(&st);
    if (rc) return rc;
    if ((rc = check_attn_tensor(q, "q")) || (rc = check_attn_tensor(k, "k")) || (rc = check_attn_tensor(v, "v")) ||
        (rc = check_attn_tensor(out, "out")) || (rc = check_attn_tensor(dout, "dout")))
        return rc;
    if (params == nullptr || dq == nullptr || dk == nullptr || dv == nullptr)
        return fail(ADA_ERR_INVALID, "null argument");
    const int64_t B = q->shape[0], H = q->shape[1], Nq = q->shape[2], Dqk = q->shape[3];
    const int64_t Nk = k->shape[2], Dv = v->shape[3];
    const AdaTensor* bh_views[4] = {k, v, out, dout};
    for (const AdaTensor* t : bh_views)
        if (t->shape[0] != B || t->shape[1] != H) return fail(ADA_ERR_SHAPE, "batch/head extents differ");
    if (k->shape[3] != Dqk || v->shape[2] != Nk) return fail(ADA_ERR_SHAPE, "k must be [B,H,Nk,Dqk], v [B,H,Nk,Dv]");
    if (out->shape[2] != Nq || out->shape[3] != Dv || dout->shape[2] != Nq || dout->shape[3] != Dv)
        return fail(ADA_ERR_SHAPE, "out and dout must be [B,H,Nq,Dv]");
    if (Dqk < 1 || Dqk > 128 || Dv < 1 || Dv > 128)
        return fail(ADA_ERR_UNSUPPORTED, "backward head dims must lie in [1, 128]");
    // gradients: fp32, contiguous [B,H,N,D]
    auto grad_ok = [](const AdaTensor* g, int64_t b, int64_t h, int64_t n, int64_t d) {
        if (g->data == nullptr || g->dtype != ADA_F32 || g->ndim != 4) return false;
        const int64_t want[4] = {b, h, n, d};
        const int64_t stride[4] = {h * n * d, n * d, d, 1};
        for (int i = 0; i < 4; ++i) {
            if (g->shape[i] != want[i]) return false;
            if (want[i] > 1 && g->stride[i] != stride[i]) return false;
        }
        return true;
    };
    if (!grad_ok(dq, B, H, Nq, Dqk) || !grad_ok(dk, B, H, Nk, Dqk) || !grad_ok(dv, B, H, Nk, Dv))
        return fail(ADA_ERR_LAYOUT, "dq, dk, dv must be contiguous fp32 [B,H,N,D] tensors");
    if (mask != nullptr && mask->data != nullptr) {
        if (mask->ndim != 4) return fail(ADA_ERR_SHAPE, "mask must be a 4-D [B,H,Nq,Nk] view");
        if (mask->dtype != ADA_BOOL && !is_float(mask->dtype)) return fail(ADA_ERR_DTYPE, "mask dtype");
        const int64_t want[4] = {B, H, Nq, Nk};
        for (int i = 0; i < 4; ++i)
            if (mask->shape[i] != want[i] && mask->shape[i] != 1) return fail(ADA_ERR_SHAPE, "mask extents");
    }
    if (B * H == 0 || Nq == 0 || Nk == 0) return ADA_OK;
    if (workspace == nullptr || workspace_bytes < ada_attn_bwd_workspace_bytes(B, H, Nq))
        return fail(ADA_ERR_WORKSPACE, "backward workspace too small");
    BwdLaunch L{};
    L.q = q->data;
    L.k = k->data;
    L.v = v->data;
    L.out = out->data;
    L.dout = dout->data;
    L.q_dtype = q->dtype;
    L.k_dtype = k->dtype;
    L.v_dtype = v->dtype;
    L.out_dtype = out->dtype;
    L.dout_dtype = dout->dtype;
    copy_strides(L.qs, q);
    copy_strides(L.ks, k);
    copy_strides(L.vs, v);
    copy_strides(L.os, out);
    copy_strides(L.gs, dout);
    L.B = B;
    L.H = H;
    L.Nq = Nq;
    L.Nk = Nk;
    L.dqk = static_cast<int>(Dqk);
    L.dv = static_cast<int>(Dv);
    L.scale = params->scale;
    L.causal = params->causal;
    L.mask = mask_view(mask);
    L.sel = HeadSelect{decisions, 0x1Fu, low_rank};
    const size_t half = ada_attn_bwd_workspace_bytes(B, H, Nq) / 2;
    L.lse = static_cast<float*>(workspace);
    L.delta = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + half);
    L.dq = static_cast<float*>(dq->data);
    L.dk = static_cast<float*>(dk->data);
    L.dv_out = static_cast<float*>(dv->data);
    rc = launch_attn_bwd(L, static_cast<cudaStream_t>(stream));
    return rc ? fail(rc, "backward launch failed: %s", cudaGetErrorString(cudaGetLastError())) : ADA_OK;
}

int ada_linear(const AdaTensor* x, const AdaTensor* w, const AdaTensor* bias, const AdaTensor* residual,
               int32_t activation, AdaTensor* y, void* stream) {
    unsigned int* st;
    int rc = device_setup(&st);
    if (rc) return rc;
    if (x == nullptr || w == nullptr || y == nullptr) return fail(ADA_ERR_INVALID, "x, w and y must be non-null");
    if (x->ndim != 2 || w->ndim != 2 || y->ndim != 2)
        return fail(ADA_ERR_SHAPE, "x [M,K], w [N,K] and y [M,N] must be 2-D");
    const int dt = x->dtype;
    if (dt != ADA_BF16 && dt != ADA_F16) return fail(ADA_ERR_DTYPE, "x must be bf16 or fp16");
    if (w->dtype != dt || y->dtype != dt) return fail(ADA_ERR_DTYPE, "x, w and y must share one dtype");
    const int64_t M = x->shape[0], K = x->shape[1], N = w->shape[0];
    if (M < 0 || K < 0 || N < 0) return fail(ADA_ERR_SHAPE, "negative extent");
    if (w->shape[1] != K) return fail(ADA_ERR_SHAPE, "w must be [N, K] with K = x.shape[1]");
    if (y->shape[0] != M || y->shape[1] != N) return fail(ADA_ERR_SHAPE, "y must be [M, N]");
    if (activation != 0 && activation != 1) return fail(ADA_ERR_INVALID, "activation must be 0 (none) or 1 (gelu)");
    if (bias != nullptr && bias->data != nullptr) {
        if (bias->dtype != dt) return fail(ADA_ERR_DTYPE, "bias dtype differs from x");
        if (bias->ndim != 1 || bias->shape[0] != N || (N > 1 && bias->stride[0] != 1))
            return fail(ADA_ERR_SHAPE, "bias must be a contiguous [N] vector");
    }
    const bool has_r = residual != nullptr && residual->data != nullptr;
    if (has_r) {
        if (residual->dtype != dt) return fail(ADA_ERR_DTYPE, "residual dtype differs from x");
        if (residual->ndim != 2 || residual->shape[0] != M || residual->shape[1] != N)
            return fail(ADA_ERR_SHAPE, "residual must be [M, N]");
    }
    if (M == 0 || N == 0) return ADA_OK;
    if (K == 0) return fail(ADA_ERR_UNSUPPORTED, "K = 0");
    if (x->data == nullptr || w->data == nullptr || y->data == nullptr)
        return fail(ADA_ERR_INVALID, "x, w and y data must be non-null");
    // TMA: 16-byte aligned bases and row strides, unit inner strides.
    auto rows_ok = [](const AdaTensor* t) {
        return aligned16(t->data) && (t->shape[1] <= 1 || t->stride[1] == 1) &&
               (t->shape[0] <= 1 || (t->stride[0] > 0 && (t->stride[0] * 2) % 16 == 0));
    };
    if (!rows_ok(x) || !rows_ok(w))
        return fail(ADA_ERR_LAYOUT, "x and w need unit column strides, 16-byte aligned bases and row strides");
    if (N > 1 && y->stride[1] != 1) return fail(ADA_ERR_LAYOUT, "y needs a unit column stride");
    if (has_r && N > 1 && residual->stride[1] != 1) return fail(ADA_ERR_LAYOUT, "residual needs a unit column stride");
    if (M >= (int64_t(1) << 31) || N >= (int64_t(1) << 31) || K >= (int64_t(1) << 31))
        return fail(ADA_ERR_UNSUPPORTED, "extents must be below 2^31");
    LinearLaunch L{};
    const CUtensorMapDataType tdt = tma_dtype(dt);
    if ((rc = make_map_rows(&L.tx, x->data, tdt, K, M, x->stride[0], 128)) ||
        (rc = make_map_rows(&L.tw, w->data, tdt, K, N, w->stride[0], 128)))
        return rc;
    L.bias = (bias != nullptr) ? bias->data : nullptr;
    L.resid = has_r ? residual->data : nullptr;
    L.n_fastest = M >= N ? 1 : 0;  // x (M x K) is the larger operand: read it once
    L.y = y->data;
    L.M = M;
    L.N = N;
    L.K = K;
    L.ld_y = M > 1 ? y->stride[0] : N;
    L.ld_r = has_r ? (M > 1 ? residual->stride[0] : N) : 0;
    L.dtype = dt;
    L.act = activation;
    const bool bias_vec = L.bias == nullptr || aligned16(L.bias);
    const bool r_vec = !has_r || (aligned16(L.resid) && (L.ld_r * 2) % 16 == 0);
    (void)bias_vec;
    L.vec = (aligned16(L.y) && (L.ld_y * 2) % 16 == 0 && r_vec) ? 1 : 0;
    // Output (and residual) tiles through TMA when their rows are 16-byte aligned.
    L.tma_io = L.vec;
    if (L.tma_io) {
        if ((rc = make_map_rows(&L.ty, L.y, tdt, N, M, L.ld_y, 32))) return rc;
        if (has_r && (rc = make_map_rows(&L.tr, L.resid, tdt, N, M, L.ld_r, 32))) return rc;
    }
    L.status = st;
    L.timeout_ns = wait_timeout_ns();
    rc = launch_linear_tc(L, static_cast<cudaStream_t>(stream));
    return rc ? fail(rc, "linear launch failed: %s", cudaGetErrorString(cudaGetLastError())) : ADA_OK;
}

int ada_layer_norm(const AdaTensor* x, const AdaTensor* weight, const AdaTensor* bias, float eps, AdaTensor* y,
                   void* stream) {
    unsigned int* st;
    int rc = device_setup(&st);
    if (rc) return rc;
    if (x == nullptr || y == nullptr) return fail(ADA_ERR_INVALID, "x and y must be non-null");
    if (x->ndim != 2 || y->ndim != 2) return fail(ADA_ERR_SHAPE, "x and y must be 2-D [M, E]");
    const int dt = x->dtype;
    if (dt != ADA_BF16 && dt != ADA_F16) return fail(ADA_ERR_DTYPE, "x must be bf16 or fp16");
    if (y->dtype != dt) return fail(ADA_ERR_DTYPE, "y dtype differs from x");
    const int64_t M = x->shape[0], E = x->shape[1];
    if (y->shape[0] != M || y->shape[1] != E) return fail(ADA_ERR_SHAPE, "y must be [M, E]");
    const AdaTensor* params[2] = {weight, bias};
    for (const AdaTensor* t : params) {
        if (t == nullptr || t->data == nullptr) continue;
        if (t->dtype != dt) return fail(ADA_ERR_DTYPE, "weight and bias must have x's dtype");
        if (t->ndim != 1 || t->shape[0] != E || (E > 1 && t->stride[0] != 1) || !aligned16(t->data))
            return fail(ADA_ERR_LAYOUT, "weight and bias must be contiguous, 16-byte aligned [E] vectors");
    }
    if (M == 0) return ADA_OK;
    if (E <= 0 || E % 8 != 0 || E > 2048) return fail(ADA_ERR_UNSUPPORTED, "E must be a multiple of 8 in [8, 2048]");
    auto rows_ok = [](const AdaTensor* t) {
        return t->data != nullptr && aligned16(t->data) && t->stride[1] == 1 &&
               (t->shape[0] <= 1 || (t->stride[0] * 2) % 16 == 0);
    };
    if (!rows_ok(x) || !rows_ok(y))
        return fail(ADA_ERR_LAYOUT, "x and y need unit column strides and 16-byte aligned rows");
    NormLaunch L{};
    L.x = x->data;
    L.y = y->data;
    L.weight = (weight != nullptr) ? weight->data : nullptr;
    L.bias = (bias != nullptr) ? bias->data : nullptr;
    L.M = M;
    L.E = static_cast<int>(E);
    L.ld_x = M > 1 ? x->stride[0] : E;
    L.ld_y = M > 1 ? y->stride[0] : E;
    L.dtype = dt;
    L.eps = eps;
    rc = launch_layer_norm(L, static_cast<cudaStream_t>(stream));
    return rc ? fail(rc, "layer-norm launch failed") : ADA_OK;
}

int ada_record_statistics(const float* summary, AdaTensor* call_count, AdaTensor* low_rank_calls,
                          AdaTensor* precision_distribution, void* stream) {
    unsigned int* st;
    int rc = device_setup(&st);
    if (rc) return rc;
    if (summary == nullptr || call_count == nullptr || low_rank_calls == nullptr || precision_distribution == nullptr ||
        call_count->data == nullptr || low_rank_calls->data == nullptr || precision_distribution->data == nullptr)
        return fail(ADA_ERR_INVALID, "null argument");
    if (call_count->dtype != ADA_I64) return fail(ADA_ERR_DTYPE, "call_count must be int64");
    auto float_ok = [](int d) { return d == ADA_F32 || d == ADA_F16 || d == ADA_BF16 || d == ADA_F64; };
    if (!float_ok(low_rank_calls->dtype) || !float_ok(precision_distribution->dtype))
        return fail(ADA_ERR_DTYPE, "statistics buffers must be floating point");
    if (precision_distribution->ndim != 1 || precision_distribution->shape[0] != 4 ||
        precision_distribution->stride[0] != 1)
        return fail(ADA_ERR_SHAPE, "precision_distribution must be a contiguous [4] vector");
    rc = launch_record_stats(summary, static_cast<int64_t*>(call_count->data), low_rank_calls->data,
                             low_rank_calls->dtype, precision_distribution->data, precision_distribution->dtype,
                             static_cast<cudaStream_t>(stream));
    return rc ? fail(rc, "statistics launch failed") : ADA_OK;
}

int ada_debug_bounded_wait(uint64_t timeout_ns, void* stream) {
    unsigned int* st;
    int rc = device_setup(&st);
    if (rc) return rc;
    rc = launch_bounded_wait(timeout_ns, st, static_cast<cudaStream_t>(stream));
    return rc ? fail(rc, "bounded-wait launch failed") : ADA_OK;
}

}  // extern "C"
