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
#include "quant_common.cuh"

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

// ---------------------------------------------------------------------------
// 16-byte variant (D % 8 == 0): 64 threads per row.  Physical thread p holds the
// two 4-element "virtual threads" 2p and 2p+1 of the 128-thread geometry above:
// its 16-byte vector it*64 + p is exactly the 4-element vectors it*128 + 2p and
// it*128 + 2p + 1.  Each virtual thread keeps its own accumulator (acc0 / acc1),
// so the per-thread FMA order is unchanged; the virtual shuffle-down tree
// 16, 8, 4, 2, 1 becomes physical shuffles 8, 4, 2, 1 inside 16-lane groups
// followed by acc0 + acc1, and the four virtual warp sums sit at lanes 0 and 16
// of the two physical warps.  Conversions to bf16 are paired
// (cvt.rn.bf16x2.f32).  Q8 emits the row's int8 codes and fp32 scale instead of
// h (the quantiser fused into its producer).
constexpr int kNorm8Threads = 64;

// The bf16 pair of a 32-bit word as an f32x2 operand (lane 0 = bits 0-15).
__device__ __forceinline__ uint64_t bf2(uint32_t v) { return f2(bf16_lo(v), bf16_hi(v)); }

// bf16 pair from an f32x2 value, each lane rounded to nearest even
__device__ __forceinline__ uint32_t rbf2(uint64_t v) {
    float a, b;
    f2_split(v, a, b);
    return pack_bf16x2(a, b);
}

// The per-element arithmetic below runs on fp32 pairs (f32x2 instructions
// round each lane exactly as the scalar __fmul_rn / __fadd_rn would), two
// elements per instruction; the rounding points are unchanged.
__device__ __forceinline__ uint32_t norm2(uint32_t xp, uint64_t rstd2, uint32_t wp, uint32_t sp, uint32_t hp) {
    const uint32_t y = rbf2(mul2(bf2(wp), mul2(rstd2, bf2(xp))));
    const uint32_t z = rbf2(mul2(bf2(y), bf2(sp)));
    return rbf2(add2(bf2(z), bf2(hp)));
}

// Plain RMSNorm with weight (no modulation): rbf16(w * (rstd * x)), the first
// rounding point of norm2 -- F.rms_norm's output.
__device__ __forceinline__ uint32_t rms2(uint32_t xp, uint64_t rstd2, uint32_t wp) {
    return rbf2(mul2(bf2(wp), mul2(rstd2, bf2(xp))));
}

// x + o * g: the bf16 product is exact in fp32, the sum rounds once (gate1)
__device__ __forceinline__ uint32_t gate2(uint32_t xp, uint32_t op, uint32_t gp) {
    return rbf2(add2(bf2(xp), mul2(bf2(op), bf2(gp))));
}

__device__ __forceinline__ float sumsq2(uint32_t v, float acc) {
    const float a = bf16_lo(v), b = bf16_hi(v);
    acc = __fmaf_rn(a, a, acc);
    return __fmaf_rn(b, b, acc);
}

template <int IT, bool GATE, bool Q8>
__global__ void __launch_bounds__(kNorm8Threads) norm8_kernel(NormArgs a, int8_t* __restrict__ xq,
                                                              float* __restrict__ xs) {
    const int64_t row = blockIdx.x;
    const int p = threadIdx.x, lane = p & 31, warp = p >> 5;
    const int r = a.ridx ? a.ridx[row] : 0;  // no table index: plain RMSNorm (s1 == sh == NULL)
    const int nv = a.D >> 3;
    uint4* xr = reinterpret_cast<uint4*>(a.x + row * (int64_t)a.D);
    // The row's loads do not depend on its table index: issue them before the
    // index load completes (the index only selects the modulation rows).
    uint4 v[IT];
#pragma unroll
    for (int it = 0; it < IT; ++it) {
        const int j = it * kNorm8Threads + p;
        if (j < nv) v[it] = xr[j];
    }
    uint4 ov[GATE ? IT : 1];
    if constexpr (GATE) {
        const uint4* orow = reinterpret_cast<const uint4*>(a.o + row * (int64_t)a.D);
#pragma unroll
        for (int it = 0; it < IT; ++it) {
            const int j = it * kNorm8Threads + p;
            if (j < nv) ov[it] = orow[j];
        }
    }
    if (r < 0 || r >= a.R) {
        if (p == 0) report(a.status, H3B_STATUS_BAD_INDEX);
        return;
    }
    if constexpr (GATE) {
        const uint4* grow = reinterpret_cast<const uint4*>(a.g + (int64_t)r * a.D);
#pragma unroll
        for (int it = 0; it < IT; ++it) {
            const int j = it * kNorm8Threads + p;
            if (j < nv) {
                const uint4 o4 = ov[it], g4 = grow[j];
                v[it] = make_uint4(gate2(v[it].x, o4.x, g4.x), gate2(v[it].y, o4.y, g4.y), gate2(v[it].z, o4.z, g4.z),
                                   gate2(v[it].w, o4.w, g4.w));
                xr[j] = v[it];
            }
        }
    }
    float acc0 = 0.0f, acc1 = 0.0f;
#pragma unroll
    for (int it = 0; it < IT; ++it) {
        const int j = it * kNorm8Threads + p;
        if (j < nv) {
            acc0 = sumsq2(v[it].y, sumsq2(v[it].x, acc0));
            acc1 = sumsq2(v[it].w, sumsq2(v[it].z, acc1));
        }
    }
#pragma unroll
    for (int off = 8; off >= 1; off >>= 1) {
        acc0 = __fadd_rn(acc0, __shfl_down_sync(0xffffffffu, acc0, off, 16));
        acc1 = __fadd_rn(acc1, __shfl_down_sync(0xffffffffu, acc1, off, 16));
    }
    __shared__ float wsum[4];
    __shared__ uint32_t wmax[2];
    if ((lane & 15) == 0) wsum[warp * 2 + (lane >> 4)] = __fadd_rn(acc0, acc1);
    __syncthreads();
    const float tot = __fadd_rn(__fadd_rn(wsum[0], wsum[2]), __fadd_rn(wsum[1], wsum[3]));
    const float rstd = rsqrtf(__fadd_rn(__fdiv_rn(tot, (float)a.D), a.eps));
    const uint64_t rstd2 = f2(rstd, rstd);

    const uint4* wv = reinterpret_cast<const uint4*>(a.w);
    const bool modulate = a.s1 != nullptr;
    const uint4* s1r = reinterpret_cast<const uint4*>(a.s1 + (int64_t)r * a.D);
    const uint4* shr = reinterpret_cast<const uint4*>(a.sh + (int64_t)r * a.D);
    uint4* hr = reinterpret_cast<uint4*>(a.h + row * (int64_t)a.D);
    uint32_t m = 0;
#pragma unroll
    for (int it = 0; it < IT; ++it) {
        const int j = it * kNorm8Threads + p;
        if (j < nv) {
            const uint4 w4 = wv[j];
            uint4 y;
            if (modulate) {
                const uint4 s4 = s1r[j], h4 = shr[j];
                y = make_uint4(norm2(v[it].x, rstd2, w4.x, s4.x, h4.x), norm2(v[it].y, rstd2, w4.y, s4.y, h4.y),
                               norm2(v[it].z, rstd2, w4.z, s4.z, h4.z), norm2(v[it].w, rstd2, w4.w, s4.w, h4.w));
            } else {
                y = make_uint4(rms2(v[it].x, rstd2, w4.x), rms2(v[it].y, rstd2, w4.y), rms2(v[it].z, rstd2, w4.z),
                               rms2(v[it].w, rstd2, w4.w));
            }
            if constexpr (Q8) {
                v[it] = y;
                m = absmax_bits8(y, m);
            } else {
                hr[j] = y;
            }
        }
    }
    if constexpr (Q8) {
        uint32_t mb = __reduce_max_sync(0xffffffffu, max(m & 0xFFFFu, m >> 16));
        if (lane == 0) wmax[warp] = mb;
        __syncthreads();
        mb = max(wmax[0], wmax[1]);
        float sc, rc;
        row_scale(__uint_as_float(mb << 16), sc, rc);
        if (p == 0) xs[row] = sc;
        uint2* qr = reinterpret_cast<uint2*>(xq + row * (int64_t)a.D);
#pragma unroll
        for (int it = 0; it < IT; ++it) {
            const int j = it * kNorm8Threads + p;
            if (j < nv) {
                float f[8];
                unpack8(v[it], f);
                qr[j] = quant8(f, sc, rc);
            }
        }
    }
}

template <bool GATE, bool Q8>
static int launch_norm8(const NormArgs& a, int64_t S, int8_t* xq, float* xs, cudaStream_t s) {
    const int need = (a.D / 8 + kNorm8Threads - 1) / kNorm8Threads;
    static const int opts[] = {1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13, 14, 15, 16, 20, 24, 28, 32};
    int it = -1;
    for (int o : opts)
        if (o >= need) {
            it = o;
            break;
        }
    dim3 grid((unsigned)S), block(kNorm8Threads);
    switch (it) {
#define H3B_N8(I) \
    case I: norm8_kernel<I, GATE, Q8><<<grid, block, 0, s>>>(a, xq, xs); break;
        H3B_N8(1) H3B_N8(2) H3B_N8(3) H3B_N8(4) H3B_N8(5) H3B_N8(6) H3B_N8(7) H3B_N8(8) H3B_N8(9) H3B_N8(10)
        H3B_N8(11) H3B_N8(12) H3B_N8(13) H3B_N8(14) H3B_N8(15) H3B_N8(16) H3B_N8(20) H3B_N8(24) H3B_N8(28) H3B_N8(32)
#undef H3B_N8
        default: return set_error(H3B_ERR_UNSUPPORTED, "norm kernels: D=%d exceeds 16384", a.D);
    }
    H3B_CUDA_TRY(cudaGetLastError());
    return H3B_OK;
}

static bool norm8_ok(const NormArgs& a) {
    return a.D % 8 == 0 && aligned(a.x, 16) && aligned(a.w, 16) && aligned(a.s1, 16) && aligned(a.sh, 16) &&
           (!a.h || aligned(a.h, 16)) && (!a.o || aligned(a.o, 16)) && (!a.g || aligned(a.g, 16));
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
    if (norm8_ok(a)) return launch_norm8<false, false>(a, S, nullptr, nullptr, static_cast<cudaStream_t>(stream));
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
    if (norm8_ok(a)) return launch_norm8<true, false>(a, S, nullptr, nullptr, static_cast<cudaStream_t>(stream));
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

extern "C" int h3b_norm_mod_quant(const void* x, const void* w, float eps, const int32_t* ridx, const void* s1,
                                  const void* sh, int8_t* xq, float* xs, int64_t S, int64_t D, int64_t R,
                                  void* stream) {
    if (int rc = check_common(x, w, ridx, s1, sh, xq, S, D, R, "h3b_norm_mod_quant")) return rc;
    H3B_REQUIRE(xs != nullptr, "h3b_norm_mod_quant: xs is NULL");
    if (S == 0) return H3B_OK;
    DeviceStatus ds;
    if (int rc = device_status(&ds)) return rc;
    NormArgs a{const_cast<uint16_t*>(static_cast<const uint16_t*>(x)), nullptr, nullptr,
               static_cast<const uint16_t*>(w), ridx, static_cast<const uint16_t*>(s1),
               static_cast<const uint16_t*>(sh), nullptr, eps, (int)D, (int)R, ds.word};
    H3B_REQUIRE(norm8_ok(a), "h3b_norm_mod_quant: needs D %% 8 == 0 and 16-byte aligned tensors");
    return launch_norm8<false, true>(a, S, xq, xs, static_cast<cudaStream_t>(stream));
}

extern "C" int h3b_gate_norm_mod_quant_(void* x, const void* o, const void* g, const void* w, float eps,
                                        const int32_t* ridx, const void* s1, const void* sh, int8_t* xq, float* xs,
                                        int64_t S, int64_t D, int64_t R, void* stream) {
    if (int rc = check_common(x, w, ridx, s1, sh, xq, S, D, R, "h3b_gate_norm_mod_quant_")) return rc;
    H3B_REQUIRE(o && g && xs, "h3b_gate_norm_mod_quant_: NULL pointer");
    if (S == 0) return H3B_OK;
    DeviceStatus ds;
    if (int rc = device_status(&ds)) return rc;
    NormArgs a{static_cast<uint16_t*>(x), static_cast<const uint16_t*>(o), static_cast<const uint16_t*>(g),
               static_cast<const uint16_t*>(w), ridx, static_cast<const uint16_t*>(s1),
               static_cast<const uint16_t*>(sh), nullptr, eps, (int)D, (int)R, ds.word};
    H3B_REQUIRE(norm8_ok(a), "h3b_gate_norm_mod_quant_: needs D %% 8 == 0 and 16-byte aligned tensors");
    return launch_norm8<true, true>(a, S, xq, xs, static_cast<cudaStream_t>(stream));
}

extern "C" int h3b_rms_norm(const void* x, const void* w, float eps, void* h, int64_t S, int64_t D, void* stream) {
    H3B_REQUIRE(x && w && h, "h3b_rms_norm: NULL pointer");
    H3B_REQUIRE(S >= 0 && S < (1ll << 31), "h3b_rms_norm: bad S=%lld", (long long)S);
    H3B_REQUIRE(D > 0 && D % 8 == 0 && D <= 16384, "h3b_rms_norm: D=%lld must be a positive multiple of 8 <= 16384",
                (long long)D);
    if (S == 0) return H3B_OK;
    DeviceStatus ds;
    if (int rc = device_status(&ds)) return rc;
    NormArgs a{const_cast<uint16_t*>(static_cast<const uint16_t*>(x)), nullptr, nullptr, static_cast<const uint16_t*>(w),
               nullptr, nullptr, nullptr, static_cast<uint16_t*>(h), eps, (int)D, 1, ds.word};
    H3B_REQUIRE(norm8_ok(a), "h3b_rms_norm: x, w and h must be 16-byte aligned");
    return launch_norm8<false, false>(a, S, nullptr, nullptr, static_cast<cudaStream_t>(stream));
}
