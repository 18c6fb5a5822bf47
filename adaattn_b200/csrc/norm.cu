// The host transformer block's LayerNorms (examples/transformer_integration.py:
// 44-45, 81: nn.LayerNorm over the embedding), which sit between the
// attention module's out_proj and the next layer's q/k/v projection, and the
// module's running decision statistics (src/adaattn/attention/adaattn.py:
// 486-498: call count, low-rank ratio, precision distribution).
//
// LayerNorm: one warp per row, the row held in registers as packed 16-bit
// pairs (16-byte loads, E <= 32 * 8 * kMaxChunks), mean and variance in fp32
// from two passes over the registers (no cancellation from E[x^2] - E[x]^2),
// y = (x - mean) * rsqrt(var + eps) * weight + bias rounded once to the
// dtype: PyTorch's fp32 arithmetic for 16-bit LayerNorm. HBM-bound: each row
// is read once and written once.
#include "ada_common.cuh"
#include "ada_internal.h"

namespace ada {
namespace {

constexpr int kNormWarps = 8;
constexpr int kMaxChunks = 8;  // 16-byte chunks per lane: E <= 2048

template <int DT>
__device__ __forceinline__ void unpack2(uint32_t v, float& lo, float& hi) {
    if constexpr (DT == ADA_BF16) {
        lo = __uint_as_float(v << 16);
        hi = __uint_as_float(v & 0xFFFF0000u);
    } else {
        unpack_f16x2(v, lo, hi);
    }
}

template <int DT>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    if constexpr (DT == ADA_BF16) return pack_bf16x2(lo, hi);
    else return pack_f16x2(lo, hi);
}

template <int DT, int CH>
__global__ void __launch_bounds__(kNormWarps * 32) layer_norm_kernel(const NormLaunch L) {
    const int lane = threadIdx.x & 31;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * kNormWarps + (threadIdx.x >> 5);
    if (row >= L.M) return;
    const int E = L.E;
    const uint4* xr = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(L.x) + row * L.ld_x);
    uint4 v[CH];
    float sum = 0.f;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
        const int col = (c * 32 + lane) * 8;
        v[c] = col < E ? xr[c * 32 + lane] : make_uint4(0, 0, 0, 0);
        const uint32_t w[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            float a, b;
            unpack2<DT>(w[e], a, b);
            sum += a + b;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float mean = sum / static_cast<float>(E);
    float sq = 0.f;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
        const int col = (c * 32 + lane) * 8;
        if (col >= E) continue;
        const uint32_t w[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            float a, b;
            unpack2<DT>(w[e], a, b);
            a -= mean;
            b -= mean;
            sq += a * a + b * b;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    const float rstd = rsqrtf(sq / static_cast<float>(E) + L.eps);
    const uint4* gw = reinterpret_cast<const uint4*>(L.weight);
    const uint4* gb = reinterpret_cast<const uint4*>(L.bias);
    uint4* yr = reinterpret_cast<uint4*>(static_cast<uint16_t*>(L.y) + row * L.ld_y);
#pragma unroll
    for (int c = 0; c < CH; ++c) {
        const int col = (c * 32 + lane) * 8;
        if (col >= E) continue;
        const uint4 wv = gw != nullptr ? __ldg(gw + c * 32 + lane) : make_uint4(0, 0, 0, 0);
        const uint4 bv = gb != nullptr ? __ldg(gb + c * 32 + lane) : make_uint4(0, 0, 0, 0);
        const uint32_t xw[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
        const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
        const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w};
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            float x0, x1, w0 = 1.f, w1 = 1.f, b0 = 0.f, b1 = 0.f;
            unpack2<DT>(xw[e], x0, x1);
            if (gw != nullptr) unpack2<DT>(ww[e], w0, w1);
            if (gb != nullptr) unpack2<DT>(bw[e], b0, b1);
            o[e] = pack2<DT>((x0 - mean) * rstd * w0 + b0, (x1 - mean) * rstd * w1 + b1);
        }
        yr[c * 32 + lane] = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

template <int DT>
int launch_norm_dt(const NormLaunch& L, cudaStream_t stream) {
    const int ch = (L.E + 255) / 256;
    const unsigned grid = static_cast<unsigned>((L.M + kNormWarps - 1) / kNormWarps);
    switch (ch) {
#define ADA_NORM_CASE(n) \
    case n: layer_norm_kernel<DT, n><<<grid, kNormWarps * 32, 0, stream>>>(L); break;
        ADA_NORM_CASE(1)
        ADA_NORM_CASE(2)
        ADA_NORM_CASE(3)
        ADA_NORM_CASE(4)
        ADA_NORM_CASE(5)
        ADA_NORM_CASE(6)
        ADA_NORM_CASE(7)
        ADA_NORM_CASE(8)
#undef ADA_NORM_CASE
        default: return ADA_ERR_UNSUPPORTED;
    }
    return cudaGetLastError() == cudaSuccess ? ADA_OK : ADA_ERR_LAUNCH;
}

// Running statistics, in the order and dtypes of the reference's updates:
// ratio = summary_count / total in fp32, cast to the buffer's dtype, then
// added in that dtype's arithmetic (fp64 for a float64 buffer, fp32 for the
// others, rounded back).
__device__ __forceinline__ void add_ratio(void* buf, int64_t i, int dtype, float ratio) {
    if (dtype == ADA_F64) {
        double* p = static_cast<double*>(buf) + i;
        *p = *p + static_cast<double>(ratio);
    } else {
        const float r = round_to(ratio, dtype);
        store_from_f32(buf, i, dtype, load_as_f32(buf, i, dtype) + r);
    }
}

__global__ void record_stats_kernel(const float* summary, int64_t* call_count, void* low_rank_calls, int lr_dtype,
                                    void* precision_distribution, int pd_dtype) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    const float total = summary[ADA_SUM_N_TOTAL];
    *call_count += 1;
    add_ratio(low_rank_calls, 0, lr_dtype, summary[ADA_SUM_N_LOWRANK] / total);
    for (int i = 0; i < 4; ++i)
        add_ratio(precision_distribution, i, pd_dtype, summary[ADA_SUM_N_FP32 + i] / total);
}

}  // namespace

int launch_layer_norm(const NormLaunch& L, cudaStream_t stream) {
    if (L.M <= 0) return ADA_OK;
    if (L.E <= 0 || L.E > 256 * kMaxChunks) return ADA_ERR_UNSUPPORTED;
    if (L.dtype == ADA_BF16) return launch_norm_dt<ADA_BF16>(L, stream);
    if (L.dtype == ADA_F16) return launch_norm_dt<ADA_F16>(L, stream);
    return ADA_ERR_DTYPE;
}

int launch_record_stats(const float* summary, int64_t* call_count, void* low_rank_calls, int lr_dtype,
                        void* precision_distribution, int pd_dtype, cudaStream_t stream) {
    record_stats_kernel<<<1, 32, 0, stream>>>(summary, call_count, low_rank_calls, lr_dtype, precision_distribution,
                                              pd_dtype);
    return cudaGetLastError() == cudaSuccess ? ADA_OK : ADA_ERR_LAUNCH;
}

}  // namespace ada
