// a4-a6: fused RMSNorm + adaLN modulation + gate/residual (HBM-bound).
//
// Bit-exactness with the reference (comfyui_nodes/h3-fuse-graph/h3_fuse_kernels.py)
// and with PyTorch's vectorized_layer_norm_kernel<bf16, float, rms=true> comes
// from keeping their reduction geometry: one row per 128-thread CTA, thread t
// owns the 4-element vectors it*128 + t (8-byte loads) and accumulates
// x*x with fused multiply-adds in (it, v) order; the four warp partials come
// from a shuffle-down tree (16, 8, 4, 2, 1) and are combined as
// (w0 + w2) + (w1 + w3).  Then var = tot / D (IEEE), rstd = rsqrtf(var + eps),
// y = bf16(w * (rstd * x)), y = bf16(y * s1[r]), h = bf16(y + sh[r]).
// The row stays in registers between the reduction and the output pass, so
// HBM sees each input byte once:
//   norm_mod       read x,   write h      4 B/element
//   gate_norm_mod_ read x,o, write x,h    8 B/element
//   gate_          read x,o, write x      6 B/element
#include "common.cuh"

namespace h3b {

constexpr int kNormThreads = 128;

struct NormArgs {
    uint16_t* x;          // [S,D] (updated in place when GATE)
    const uint16_t* o;    // [S,D] branch output (GATE only)
    const uint16_t* g;    // [R,D] gate table (GATE only)
    const uint16_t* w;    // [D]
    const int32_t* ridx;  // [S]
    const uint16_t* s1;   // [R,D]
    const uint16_t* sh;   // [R,D]
    uint16_t* h;          // [S,D]
    float eps;
    int D;
    int R;
    int* status;
};

__device__ __forceinline__ float4 unpack4(uint2 v) {
    return make_float4(bf16_lo(v.x), bf16_hi(v.x), bf16_lo(v.y), bf16_hi(v.y));
}

__device__ __forceinline__ uint2 pack4(float a, float b, float c, float d) {
    return make_uint2(pack_bf16x2(a, b), pack_bf16x2(c, d));
}

// x + o*g: o*g is exact in fp32 (bf16 operands), so this equals the GPU's fma.
__device__ __forceinline__ float gate1(float x, float o, float g) { return __fadd_rn(x, __fmul_rn(o, g)); }

__device__ __forceinline__ float norm1(float x, float rstd, float w, float s1, float sh) {
    float y = rbf16(__fmul_rn(w, __fmul_rn(rstd, x)));
    y = rbf16(__fmul_rn(y, s1));
    return __fadd_rn(y, sh);
}

template <int ITERS, bool GATE>
__global__ void __launch_bounds__(kNormThreads) norm_mod_kernel(NormArgs a) {
    const int64_t row = blockIdx.x;
    const int t = threadIdx.x;
    const int r = a.ridx[row];
    if (r < 0 || r >= a.R) {
        if (t == 0) report(a.status, H3B_STATUS_BAD_INDEX);
        return;
    }
    const int nv = a.D >> 2;  // 4-element vectors per row
    uint2* xr = reinterpret_cast<uint2*>(a.x + row * a.D);
    uint2 xv[ITERS];
    float acc = 0.0f;
#pragma unroll
    for (int it = 0; it < ITERS; ++it) {
        const int j = it * kNormThreads + t;
        if (j < nv) xv[it] = xr[j];
    }
    if constexpr (GATE) {
        const uint2* orow = reinterpret_cast<const uint2*>(a.o + row * a.D);
        const uint2* grow = reinterpret_cast<const uint2*>(a.g + (int64_t)r * a.D);
#pragma unroll
        for (int it = 0; it < ITERS; ++it) {
            const int j = it * kNormThreads + t;
            if (j < nv) {
                const float4 x4 = unpack4(xv[it]), o4 = unpack4(orow[j]), g4 = unpack4(grow[j]);
                xv[it] = pack4(gate1(x4.x, o4.x, g4.x), gate1(x4.y, o4.y, g4.y), gate1(x4.z, o4.z, g4.z),
                               gate1(x4.w, o4.w, g4.w));
                xr[j] = xv[it];
            }
        }
    }
#pragma unroll
    for (int it = 0; it < ITERS; ++it) {
        const int j = it * kNormThreads + t;
        if (j < nv) {
            const float4 x4 = unpack4(xv[it]);
            acc = __fmaf_rn(x4.x, x4.x, acc);
            acc = __fmaf_rn(x4.y, x4.y, acc);
            acc = __fmaf_rn(x4.z, x4.z, acc);
            acc = __fmaf_rn(x4.w, x4.w, acc);
        }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, off));
    __shared__ float wsum[4];
    if ((t & 31) == 0) wsum[t >> 5] = acc;
    __syncthreads();
    const float tot = __fadd_rn(__fadd_rn(wsum[0], wsum[2]), __fadd_rn(wsum[1], wsum[3]));
    const float rstd = rsqrtf(__fadd_rn(__fdiv_rn(tot, (float)a.D), a.eps));

    const uint2* wv = reinterpret_cast<const uint2*>(a.w);
    const uint2* s1r = reinterpret_cast<const uint2*>(a.s1 + (int64_t)r * a.D);
    const uint2* shr = reinterpret_cast<const uint2*>(a.sh + (int64_t)r * a.D);
    uint2* hr = reinterpret_cast<uint2*>(a.h + row * a.D);
#pragma unroll
    for (int it = 0; it < ITERS; ++it) {
        const int j = it * kNormThreads + t;
        if (j < nv) {
            const float4 x4 = unpack4(xv[it]), w4 = unpack4(wv[j]), s4 = unpack4(s1r[j]), h4 = unpack4(shr[j]);
            hr[j] = pack4(norm1(x4.x, rstd, w4.x, s4.x, h4.x), norm1(x4.y, rstd, w4.y, s4.y, h4.y),
                          norm1(x4.z, rstd, w4.z, s4.z, h4.z), norm1(x4.w, rstd, w4.w, s4.w, h4.w));
        }
    }
}

// gate_: pure elementwise, 16-byte vectors, one row per CTA.
template <bool VEC16>
__global__ void __launch_bounds__(128) gate_kernel(uint16_t* __restrict__ x, const uint16_t* __restrict__ o,
                                                   const uint16_t* __restrict__ g, const int32_t* __restrict__ ridx,
                                                   int D, int R, int* status) {
    const int64_t row = blockIdx.x;
    const int r = ridx[row];
    if (r < 0 || r >= R) {
        if (threadIdx.x == 0) report(status, H3B_STATUS_BAD_INDEX);
        return;
    }
    if constexpr (VEC16) {
        uint4* xr = reinterpret_cast<uint4*>(x + row * D);
        const uint4* orow = reinterpret_cast<const uint4*>(o + row * D);
        const uint4* grow = reinterpret_cast<const uint4*>(g + (int64_t)r * D);
        for (int j = threadIdx.x; j < (D >> 3); j += blockDim.x) {
            uint4 xv = xr[j];
            const uint4 ov = orow[j], gv = grow[j];
            uint32_t* xu = reinterpret_cast<uint32_t*>(&xv);
            const uint32_t* ou = reinterpret_cast<const uint32_t*>(&ov);
            const uint32_t* gu = reinterpret_cast<const uint32_t*>(&gv);
#pragma unroll
            for (int e = 0; e < 4; ++e)
                xu[e] = pack_bf16x2(gate1(bf16_lo(xu[e]), bf16_lo(ou[e]), bf16_lo(gu[e])),
                                    gate1(bf16_hi(xu[e]), bf16_hi(ou[e]), bf16_hi(gu[e])));
            xr[j] = xv;
        }
    } else {
        uint2* xr = reinterpret_cast<uint2*>(x + row * D);
        const uint2* orow = reinterpret_cast<const uint2*>(o + row * D);
        const uint2* grow = reinterpret_cast<const uint2*>(g + (int64_t)r * D);
        for (int j = threadIdx.x; j < (D >> 2); j += blockDim.x) {
            const float4 x4 = unpack4(xr[j]), o4 = unpack4(orow[j]), g4 = unpack4(grow[j]);
            xr[j] = pack4(gate1(x4.x, o4.x, g4.x), gate1(x4.y, o4.y, g4.y), gate1(x4.z, o4.z, g4.z),
                          gate1(x4.w, o4.w, g4.w));
        }
    }
}

template <bool GATE>
static int launch_norm(const NormArgs& a, int64_t S, cudaStream_t s) {
    const int need = (a.D / 4 + kNormThreads - 1) / kNormThreads;
    dim3 grid((unsigned)S), block(kNormThreads);
    switch (need) {
#define H3B_NCASE(I) \
    case I: norm_mod_kernel<I, GATE><<<grid, block, 0, s>>>(a); break;
        H3B_NCASE(1) H3B_NCASE(2) H3B_NCASE(3) H3B_NCASE(4) H3B_NCASE(5) H3B_NCASE(6) H3B_NCASE(7) H3B_NCASE(8)
        H3B_NCASE(9) H3B_NCASE(10) H3B_NCASE(11) H3B_NCASE(12) H3B_NCASE(13) H3B_NCASE(14) H3B_NCASE(15)
        H3B_NCASE(16) H3B_NCASE(17) H3B_NCASE(18) H3B_NCASE(19) H3B_NCASE(20) H3B_NCASE(21) H3B_NCASE(22)
        H3B_NCASE(23) H3B_NCASE(24) H3B_NCASE(25) H3B_NCASE(26) H3B_NCASE(27) H3B_NCASE(28) H3B_NCASE(29)
        H3B_NCASE(30) H3B_NCASE(31) H3B_NCASE(32)
#undef H3B_NCASE
        default: return set_error(H3B_ERR_UNSUPPORTED, "norm kernels: D=%d exceeds 16384", a.D);
    }
    H3B_CUDA_TRY(cudaGetLastError());
    return H3B_OK;
}

static int check_common(const void* x, const void* w, const int32_t* ridx, const void* s1, const void* sh,
                        const void* h, int64_t S, int64_t D, int64_t R, const char* who) {
    H3B_REQUIRE(x && w && ridx && s1 && sh && h, "%s: NULL pointer", who);
    H3B_REQUIRE(S >= 0 && S < (1ll << 31), "%s: bad S=%lld", who, (long long)S);
    H3B_REQUIRE(D > 0 && D % 4 == 0 && D <= 16384, "%s: D=%lld must be a positive multiple of 4 <= 16384", who, (long long)D);
    H3B_REQUIRE(R > 0 && R < (1ll << 31), "%s: bad R=%lld", who, (long long)R);
    H3B_REQUIRE(aligned(x, 8) && aligned(w, 8) && aligned(s1, 8) && aligned(sh, 8) && aligned(h, 8),
                "%s: tensors must be 8-byte aligned", who);
    return H3B_OK;
}

}  // namespace h3b

using namespace h3b;

extern "C" int h3b_norm_mod(const void* x, const void* w, float eps, const int32_t* ridx, const void* s1,
                            const void* sh, void* h, int64_t S, int64_t D, int64_t R, void* stream) {
    if (int rc = check_common(x, w, ridx, s1, sh, h, S, D, R, "h3b_norm_mod")) return rc;
    if (S == 0) return H3B_OK;
    DeviceStatus ds;
    if (int rc = device_status(&ds)) return rc;
    NormArgs a{const_cast<uint16_t*>(static_cast<const uint16_t*>(x)), nullptr, nullptr,
               static_cast<const uint16_t*>(w), ridx, static_cast<const uint16_t*>(s1),
               static_cast<const uint16_t*>(sh), static_cast<uint16_t*>(h), eps, (int)D, (int)R, ds.word};
    return launch_norm<false>(a, S, static_cast<cudaStream_t>(stream));
}

extern "C" int h3b_gate_norm_mod_(void* x, const void* o, const void* g, const void* w, float eps,
                                  const int32_t* ridx, const void* s1, const void* sh, void* h, int64_t S,
                                  int64_t D, int64_t R, void* stream) {
    if (int rc = check_common(x, w, ridx, s1, sh, h, S, D, R, "h3b_gate_norm_mod_")) return rc;
    H3B_REQUIRE(o && g && aligned(o, 8) && aligned(g, 8), "h3b_gate_norm_mod_: o/g NULL or misaligned");
    if (S == 0) return H3B_OK;
    DeviceStatus ds;
    if (int rc = device_status(&ds)) return rc;
    NormArgs a{static_cast<uint16_t*>(x), static_cast<const uint16_t*>(o), static_cast<const uint16_t*>(g),
               static_cast<const uint16_t*>(w), ridx, static_cast<const uint16_t*>(s1),
               static_cast<const uint16_t*>(sh), static_cast<uint16_t*>(h), eps, (int)D, (int)R, ds.word};
    return launch_norm<true>(a, S, static_cast<cudaStream_t>(stream));
}

extern "C" int h3b_gate_(void* x, const void* o, const void* g, const int32_t* ridx, int64_t S, int64_t D,
                         int64_t R, void* stream) {
    H3B_REQUIRE(x && o && g && ridx, "h3b_gate_: NULL pointer");
    H3B_REQUIRE(S >= 0 && S < (1ll << 31) && D > 0 && D % 4 == 0 && D < (1ll << 30) && R > 0,
                "h3b_gate_: bad shape S=%lld D=%lld R=%lld", (long long)S, (long long)D, (long long)R);
    H3B_REQUIRE(aligned(x, 8) && aligned(o, 8) && aligned(g, 8), "h3b_gate_: tensors must be 8-byte aligned");
    if (S == 0) return H3B_OK;
    DeviceStatus ds;
    if (int rc = device_status(&ds)) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool vec16 = D % 8 == 0 && aligned(x, 16) && aligned(o, 16) && aligned(g, 16);
    if (vec16)
        gate_kernel<true><<<(unsigned)S, 128, 0, s>>>(static_cast<uint16_t*>(x), static_cast<const uint16_t*>(o),
                                                      static_cast<const uint16_t*>(g), ridx, (int)D, (int)R, ds.word);
    else
        gate_kernel<false><<<(unsigned)S, 128, 0, s>>>(static_cast<uint16_t*>(x), static_cast<const uint16_t*>(o),
                                                       static_cast<const uint16_t*>(g), ridx, (int)D, (int)R, ds.word);
    H3B_CUDA_TRY(cudaGetLastError());
    return H3B_OK;
}
