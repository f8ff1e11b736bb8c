// a1: per-token absmax int8 quantisation of bf16 activations (HBM-bound),
// optionally fused with the GELU(tanh) that feeds the FFN down projection.
//
// One CTA per row.  The row is read once with 16-byte vector loads and held in
// registers (up to 16 vectors per thread); the absmax is an unsigned max over
// the bf16 bit patterns (warp redux + a shared-memory step, exact), then every
// element is quantised with the reciprocal fast path of quant_common.cuh.
// Bytes per row: 2K read, K + 4 written.
//
// GELU variant (h3b_gelu_quant, the input of the FFN down projection): the
// codes of bf16(gelu_tanh(x)), the value PyTorch's GeluCUDAKernelImpl computes
// in fp32 (x^3 as (x*x)*x, the inner polynomial as one fused multiply-add,
// tanhf, 0.5*x*(1+t)), so they equal quant(F.gelu(u, approximate="tanh")) bit
// for bit without the bf16 GELU output ever reaching HBM.  A bf16 input has
// 65536 values, so the GELU is a 128 KB table filled once per device by that
// formula; the kernel keeps it in shared memory and streams the rows past it
// (gelu_quant_lut_kernel below).
//
// ConvRot variant (quant_convrot_kernel): the rows are first rotated group by
// group with the Walsh-Hadamard transform, as the reference's fast path does
// before quantising (its weights are stored rotated the same way).
//
// Gather variant (the inverse Ulysses exchange fused with the quantiser of the
// attention output projection): row m is assembled from every rank's attention
// output rows, read over NVLink from the peers' buffers, so the exchanged rows
// never land in a staging buffer; codes and scales are those of the gathered
// row, bit for bit.
#include <stdlib.h>

#include <mutex>

#include "quant_common.cuh"

namespace h3b {

enum class Act { kNone = 0 };

constexpr int kMaxGatherRanks = 8;

// Row source of the inverse-exchange quantiser: vector j of local row m is
// vector j % cv of row (row0 + m) of rank j / cv's buffer src[j / cv] (rows
// ldv vectors apart; a peer's memory for the other ranks).
struct GatherRows {
    const uint4* src[kMaxGatherRanks];
    int64_t row0, ldv;
    int cv;
};

template <int VPT, int NT, Act ACT, bool GATHER>
__global__ void __launch_bounds__(NT) quant_rowwise_kernel(const uint16_t* __restrict__ x, int64_t ldx, int K,
                                                           int8_t* __restrict__ xq, float* __restrict__ xs,
                                                           const __grid_constant__ GatherRows g) {
    const int64_t row = blockIdx.x;
    const uint4* xr = reinterpret_cast<const uint4*>(x + row * ldx);
    const int nvec = K >> 3;
    uint4 v[VPT];
    uint32_t m = 0;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const int j = threadIdx.x + i * NT;
        if (j < nvec) {
            if constexpr (GATHER) {
                const int rk = j / g.cv;
                v[i] = g.src[rk][(g.row0 + row) * g.ldv + (j - rk * g.cv)];
            } else {
                v[i] = xr[j];
            }
        }
    }
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const int j = threadIdx.x + i * NT;
        if (j < nvec) {
            m = absmax_bits8(v[i], m);
        }
    }
    uint32_t mb = max(m & 0xFFFFu, m >> 16);
    mb = __reduce_max_sync(0xffffffffu, mb);
    __shared__ uint32_t wmax[NT / 32];
    if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = mb;
    __syncthreads();
    mb = wmax[0];
#pragma unroll
    for (int w = 1; w < NT / 32; ++w) mb = max(mb, wmax[w]);

    float s, r;
    row_scale(__uint_as_float(mb << 16), s, r);
    if (threadIdx.x == 0) xs[row] = s;
    uint2* qr = reinterpret_cast<uint2*>(xq + row * (int64_t)K);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const int j = threadIdx.x + i * NT;
        if (j < nvec) {
            float f[8];
            unpack8(v[i], f);
            qr[j] = quant8(f, s, r);
        }
    }
}

// ConvRot variant: each group of G columns (G = 64 or 256) of the row is rotated
// by the normalised Walsh-Hadamard transform before the absmax and the codes
// (y = H_G x / sqrt(G), Sylvester order).  Fast transform in binary32, stages
// h = 1, 2, 4 inside a thread's 8-element vector, then h = 8 .. G/2 across the
// G/8 lanes holding the group (lane ^ h/8 is the partner: the group's vectors
// sit in consecutive lanes because NT % (G/8) == 0), then the exact scale by
// 1/sqrt(G); two elements per f32x2 instruction.  Every lane runs every
// shuffle (lanes past the row's end carry zeros), so the full-warp shuffles
// never see an exited lane.
__device__ __forceinline__ uint64_t shfl_xor2(uint64_t v, int m) {
    return __shfl_xor_sync(0xffffffffu, (unsigned long long)v, m);
}

// SwiGLU input activation (the fused "swiglu" input of the reference's second
// FFN linear): the row holds 2K columns, gate a = x[:, :K], up b = x[:, K:];
// the activation bf16(silu(a) * b), silu(a) = a / (1 + expf(-a)) in fp32 with
// one rounding per operation (PyTorch's F.silu(a.float()) * b.float() cast to
// bf16), then the rotation and the codes as for a plain bf16 input.
__device__ __forceinline__ uint32_t swiglu2(uint32_t a, uint32_t b) {
    const float a0 = bf16_lo(a), a1 = bf16_hi(a);
    const float s0 = __fdiv_rn(a0, __fadd_rn(1.0f, expf(-a0)));
    const float s1 = __fdiv_rn(a1, __fadd_rn(1.0f, expf(-a1)));
    return pack_bf16x2(__fmul_rn(s0, bf16_lo(b)), __fmul_rn(s1, bf16_hi(b)));
}

template <int VPT, int NT, int G, bool SWIGLU = false>
__global__ void __launch_bounds__(NT) quant_convrot_kernel(const uint16_t* __restrict__ x, int64_t ldx, int K,
                                                           int8_t* __restrict__ xq, float* __restrict__ xs) {
    constexpr int LG = G / 8;  // lanes per group
    constexpr float kInv = G == 64 ? 0.125f : 0.0625f;
    static_assert(G == 64 || G == 256, "rotation groups of 64 or 256 columns");
    const int64_t row = blockIdx.x;
    const uint4* xr = reinterpret_cast<const uint4*>(x + row * ldx);
    const int nvec = K >> 3;
    const int lane = threadIdx.x & 31;
    // p[i][k] holds elements 2k, 2k+1 of vector i as an fp32 pair (f32x2 arithmetic)
    uint64_t p[VPT][4];
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const int j = threadIdx.x + i * NT;
        uint4 v = j < nvec ? xr[j] : make_uint4(0u, 0u, 0u, 0u);
        if constexpr (SWIGLU) {
            const uint4 u = j < nvec ? xr[nvec + j] : make_uint4(0u, 0u, 0u, 0u);
            v = make_uint4(swiglu2(v.x, u.x), swiglu2(v.y, u.y), swiglu2(v.z, u.z), swiglu2(v.w, u.w));
        }
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        // stage h = 1: pairs (2k, 2k+1) inside one word
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float a = bf16_lo(w[k]), b = bf16_hi(w[k]);
            p[i][k] = f2(__fadd_rn(a, b), __fsub_rn(a, b));
        }
        // h = 2: pairs (p0, p1), (p2, p3); h = 4: (p0, p2), (p1, p3)
        uint64_t t0 = add2(p[i][0], p[i][1]), t1 = sub2(p[i][0], p[i][1]);
        uint64_t t2 = add2(p[i][2], p[i][3]), t3 = sub2(p[i][2], p[i][3]);
        p[i][0] = add2(t0, t2);
        p[i][2] = sub2(t0, t2);
        p[i][1] = add2(t1, t3);
        p[i][3] = sub2(t1, t3);
    }
    uint32_t m = 0;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        // h = 8 .. G/2 across lanes: the lower partner takes mine + theirs, the
        // upper theirs - mine, i.e. theirs + s * mine with s = +-1 (exact product,
        // one rounding: bit-identical to the add / subtract)
#pragma unroll
        for (int sh = 1; sh < LG; sh <<= 1) {
            const float sg = (lane & sh) ? -1.0f : 1.0f;
            const uint64_t s2 = f2(sg, sg);
#pragma unroll
            for (int k = 0; k < 4; ++k) p[i][k] = fma2(s2, p[i][k], shfl_xor2(p[i][k], sh));
        }
        const uint64_t inv2 = f2(kInv, kInv);
        const int j = threadIdx.x + i * NT;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            p[i][k] = mul2(p[i][k], inv2);
            float a, b;
            f2_split(p[i][k], a, b);
            if (j < nvec) m = max(m, max(__float_as_uint(a) & 0x7FFFFFFFu, __float_as_uint(b) & 0x7FFFFFFFu));
        }
    }
    m = __reduce_max_sync(0xffffffffu, m);
    __shared__ uint32_t wmax[NT / 32];
    if (lane == 0) wmax[threadIdx.x >> 5] = m;
    __syncthreads();
    m = wmax[0];
#pragma unroll
    for (int w = 1; w < NT / 32; ++w) m = max(m, wmax[w]);
    float s, r;
    row_scale(__uint_as_float(m), s, r);
    if (threadIdx.x == 0) xs[row] = s;
    uint2* qr = reinterpret_cast<uint2*>(xq + row * (int64_t)K);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const int j = threadIdx.x + i * NT;
        if (j < nvec) {
            float f[8];
#pragma unroll
            for (int k = 0; k < 4; ++k) f2_split(p[i][k], f[2 * k], f[2 * k + 1]);
            qr[j] = quant8(f, s, r);
        }
    }
}

// Bounded mbarrier waits of the table-driven GELU kernels below.
__device__ __forceinline__ bool bar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait with a suspend-time hint: the thread sleeps in the instruction
// until the phase completes or about 0.1 ms pass, instead of spinning and
// taking issue slots from the warps that compute.
__device__ __forceinline__ bool bar_try_wait_sleep(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(100000u)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ bool bar_wait_parity_bounded(uint32_t bar, uint32_t parity, uint64_t limit_ns) {
    if (bar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        if (bar_try_wait_sleep(bar, parity)) return true;
        if (globaltimer_ns() - t0 > limit_ns) return false;
    }
}

__device__ __forceinline__ bool bar_wait_bounded(uint32_t bar, uint64_t limit_ns) {
    if (bar_try_wait(bar, 0)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t n = 1;; ++n) {
        if (bar_try_wait(bar, 0)) return true;
        if ((n & 63u) == 0 && globaltimer_ns() - t0 > limit_ns) return false;
    }
}

// ---------------------------------------------------------------------------
// GELU by table.  A bf16 -> bf16 function is determined by its 65536 outputs:
// g_gelu_table[b] = gelu2 (PyTorch's fp32 formula with tanhf) of the bf16 with
// bits b, filled once per device by gelu_table_fill_kernel from the exact
// formula, so every lookup equals F.gelu(approximate="tanh") bit for bit.
// The quantiser and the elementwise GELU keep the 128 KB table in shared
// memory (one bulk copy per CTA), one persistent CTA of 1024 threads per SM.
static __device__ __align__(128) uint16_t g_gelu_table[65536];
constexpr int kTableBytes = 65536 * 2;
constexpr int kLutThreads = 1024;
constexpr int kLutSmemMax = 227 * 1024 - 1024;  // dynamic shared memory: the table and the row buffers

__global__ void gelu_table_fill_kernel() {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;  // one bf16 pair per thread
    if (i < 32768) {
        const uint32_t v = gelu2((uint32_t)(2 * i) | ((uint32_t)(2 * i + 1) << 16));
        reinterpret_cast<uint32_t*>(g_gelu_table)[i] = v;
    }
}

// Bounded wait for the table's bulk copy (all threads); false on expiry.
__device__ __forceinline__ bool load_table(uint16_t* lut, uint64_t* bar, int* status) {
    const uint32_t sbar = (uint32_t)__cvta_generic_to_shared(bar);
    if (threadIdx.x == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(sbar) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sbar), "r"(kTableBytes) : "memory");
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                (uint32_t)__cvta_generic_to_shared(lut)),
            "l"(g_gelu_table), "r"(kTableBytes), "r"(sbar)
            : "memory");
    }
    __syncthreads();
    if (!bar_wait_bounded(sbar, 10ull * 1000 * 1000 * 1000)) {
        report(status, H3B_STATUS_MBAR_TIMEOUT);
        bar_wait_bounded(sbar, 100ull * 1000 * 1000);  // this CTA's own copy, before its shared memory goes
        return false;
    }
    return true;
}

__device__ __forceinline__ uint32_t lut2(const uint16_t* lut, uint32_t v) {
    return (uint32_t)lut[v & 0xFFFFu] | ((uint32_t)lut[v >> 16] << 16);
}

__device__ __forceinline__ uint4 lut8(const uint16_t* lut, uint4 v) {
    return make_uint4(lut2(lut, v.x), lut2(lut, v.y), lut2(lut, v.z), lut2(lut, v.w));
}

// Rows r = blockIdx.x, + gridDim.x, ...: up to kMaxRowBufs rows ahead are in
// flight as bulk copies into shared-memory row buffers (one mbarrier each),
// so the bytes in flight per SM do not depend on registers.
constexpr int kMaxRowBufs = 3;

// Two halves of 512 threads, each with its own rows (the CTA's even and odd
// rows) and its own named barrier, so one half's barrier wait is covered by
// the other half's lookups and stores.  The row buffers are shared: the half
// that releases its row k requests row k + nbuf, which may be the other
// half's.  Within a half: wait for the row's buffer, look it up, post the
// per-warp maxima, one barrier, request, scale (every warp of the half), codes.
constexpr int kHalfThreads = kLutThreads / 2;

template <int VPT>
__global__ void __launch_bounds__(kLutThreads, 1) gelu_quant_lut_kernel(const uint16_t* __restrict__ x, int64_t ldx,
                                                                           int64_t M, int K, int8_t* __restrict__ xq,
                                                                           float* __restrict__ xs, int nbuf,
                                                                           int* status) {
    extern __shared__ __align__(128) uint16_t lut[];  // 65536 table entries, then nbuf rows of K
    __shared__ __align__(8) uint64_t bar;
    __shared__ __align__(8) uint64_t full[kMaxRowBufs];
    __shared__ uint32_t wmax[2][2][kHalfThreads / 32];  // [half][row parity][warp of the half]
    const int nvec = K >> 3;
    const int t = threadIdx.x, h = t / kHalfThreads, th = t % kHalfThreads, lane = t & 31, hw = th >> 5;
    const uint32_t row_bytes = (uint32_t)K * 2u;
    uint4* rows = reinterpret_cast<uint4*>(lut + 65536);
    const int64_t step = gridDim.x;
    auto request = [&](int b, int64_t r) {  // one thread
        const uint32_t sb = (uint32_t)__cvta_generic_to_shared(&full[b]);
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sb), "r"(row_bytes) : "memory");
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                (uint32_t)__cvta_generic_to_shared(rows + (int64_t)b * nvec)),
            "l"(x + r * ldx), "r"(row_bytes), "r"(sb)
            : "memory");
    };
    if (t == 0) {
        for (int b = 0; b < nbuf; ++b)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"((uint32_t)__cvta_generic_to_shared(&full[b]))
                         : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int b = 0; b < nbuf; ++b)
            if (blockIdx.x + b * step < M) request(b, blockIdx.x + b * step);
    }
    if (!load_table(lut, &bar, status)) {
        if (t == 0)
            for (int b = 0; b < nbuf; ++b)
                if (blockIdx.x + b * step < M) bar_wait_bounded((uint32_t)__cvta_generic_to_shared(&full[b]),
                                                                100ull * 1000 * 1000);
        return;
    }
    // this half's rows: the CTA's k-th rows with k % 2 == h
    for (int k = h; blockIdx.x + k * step < M; k += 2) {
        const int64_t row = blockIdx.x + k * step;
        const int b = k % nbuf;
        if (!bar_wait_parity_bounded((uint32_t)__cvta_generic_to_shared(&full[b]), (uint32_t)((k / nbuf) & 1),
                                     10ull * 1000 * 1000 * 1000)) {
            report(status, H3B_STATUS_MBAR_TIMEOUT);
            if (th == 0)  // copies requested by this CTA that may still be in flight
                for (int j = k; j < k + nbuf && blockIdx.x + j * step < M; ++j)
                    bar_wait_parity_bounded((uint32_t)__cvta_generic_to_shared(&full[j % nbuf]),
                                            (uint32_t)((j / nbuf) & 1), 100ull * 1000 * 1000);
            return;
        }
        const uint4* rb = rows + (int64_t)b * nvec;
        uint4 v[VPT];
        uint32_t m = 0;
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
            const int j = th + i * kHalfThreads;
            if (j < nvec) {
                v[i] = lut8(lut, rb[j]);
                m = absmax_bits8(v[i], m);
            }
        }
        uint32_t mb = max(m & 0xFFFFu, m >> 16);
        mb = __reduce_max_sync(0xffffffffu, mb);
        // the maxima alternate between two slots by row, so one barrier per row
        // suffices: a warp writes slot p again two rows later, after the next
        // barrier, which every warp reaches only after reading slot p
        const int p = (k >> 1) & 1;
        if (lane == 0) wmax[h][p][hw] = mb;
        asm volatile("bar.sync %0, %1;" ::"r"(1 + h), "r"(kHalfThreads) : "memory");  // this half's row is read
        if (th == 0 && row + nbuf * step < M) request(b, row + nbuf * step);
        mb = __reduce_max_sync(0xffffffffu, wmax[h][p][lane & (kHalfThreads / 32 - 1)]);
        float s, rc;
        row_scale(__uint_as_float(mb << 16), s, rc);
        if (th == 0) xs[row] = s;
        uint2* qr = reinterpret_cast<uint2*>(xq + row * (int64_t)K);
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
            const int j = th + i * kHalfThreads;
            if (j < nvec) {
                float f[8];
                unpack8(v[i], f);
                qr[j] = quant8(f, s, rc);
            }
        }
    }
}

// Elementwise bf16 GELU by table: grid-stride over 16-byte vectors.
__global__ void __launch_bounds__(kLutThreads, 1) gelu_lut_kernel(const uint4* __restrict__ x, uint4* __restrict__ y,
                                                                    int64_t nvec, const uint32_t* __restrict__ xt,
                                                                    uint32_t* __restrict__ yt, int tail_pairs,
                                                                    int* status) {
    extern __shared__ __align__(128) uint16_t lut[];
    __shared__ __align__(8) uint64_t bar;
    const int64_t stride = (int64_t)gridDim.x * kLutThreads;
    int64_t i = (int64_t)blockIdx.x * kLutThreads + threadIdx.x;
    uint4 v = i < nvec ? x[i] : make_uint4(0u, 0u, 0u, 0u);
    if (!load_table(lut, &bar, status)) return;
    for (; i < nvec; i += stride) {
        const uint4 nv = i + stride < nvec ? x[i + stride] : make_uint4(0u, 0u, 0u, 0u);
        y[i] = lut8(lut, v);
        v = nv;
    }
    if (blockIdx.x == 0 && threadIdx.x < tail_pairs) yt[threadIdx.x] = lut2(lut, xt[threadIdx.x]);
}

// Per device, once: fill the table and allow the kernels their shared memory.
// The first call on a device launches the fill kernel on the caller's stream
// and waits for it (make that first call before any stream capture).
static int gelu_table_ready(cudaStream_t s) {
    struct Slot {
        std::once_flag once;
        cudaError_t err = cudaSuccess;
    };
    static Slot slots[64];
    int dev = 0;
    H3B_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return set_error(H3B_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
    Slot& slot = slots[dev];
    std::call_once(slot.once, [&slot, s] {
        cudaError_t e = cudaFuncSetAttribute(gelu_lut_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kTableBytes);
        for (auto fn : {gelu_quant_lut_kernel<1>, gelu_quant_lut_kernel<2>, gelu_quant_lut_kernel<4>,
                        gelu_quant_lut_kernel<8>})
            if (e == cudaSuccess) e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kLutSmemMax);
        if (e == cudaSuccess) {
            gelu_table_fill_kernel<<<128, 256, 0, s>>>();
            e = cudaGetLastError();
        }
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        slot.err = e;
    });
    if (slot.err != cudaSuccess) return cuda_error(slot.err, "GELU table set-up");
    return H3B_OK;
}

static int num_sms_here() {
    int dev = 0, n = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
}

static int gelu_quant_lut(const uint16_t* x, int64_t ldx, int64_t M, int K, int8_t* xq, float* xs, cudaStream_t s) {
    if (int rc = gelu_table_ready(s)) return rc;
    DeviceStatus ds;
    if (int rc = device_status(&ds)) return rc;
    const int nvec = K / 8;
    const int row_bytes = K * 2;
    int nbuf = (kLutSmemMax - kTableBytes) / row_bytes;  // >= 1 for K <= 32768
    if (nbuf > kMaxRowBufs) nbuf = kMaxRowBufs;
    const int smem = kTableBytes + nbuf * row_bytes;
    const int64_t sms = num_sms_here();
    const unsigned grid = (unsigned)(M < sms ? M : sms);
    const int v2 = (nvec + kHalfThreads - 1) / kHalfThreads;  // vectors per thread, <= 8 for K <= 32768
    if (v2 <= 1) gelu_quant_lut_kernel<1><<<grid, kLutThreads, smem, s>>>(x, ldx, M, K, xq, xs, nbuf, ds.word);
    else if (v2 <= 2) gelu_quant_lut_kernel<2><<<grid, kLutThreads, smem, s>>>(x, ldx, M, K, xq, xs, nbuf, ds.word);
    else if (v2 <= 4) gelu_quant_lut_kernel<4><<<grid, kLutThreads, smem, s>>>(x, ldx, M, K, xq, xs, nbuf, ds.word);
    else gelu_quant_lut_kernel<8><<<grid, kLutThreads, smem, s>>>(x, ldx, M, K, xq, xs, nbuf, ds.word);
    H3B_CUDA_TRY(cudaGetLastError());
    return H3B_OK;
}

template <int NT, int G, bool SWIGLU>
static void launch_convrot(int vpt, const uint16_t* x, int64_t ldx, int64_t M, int K, int8_t* xq, float* xs,
                           cudaStream_t s) {
    dim3 grid((unsigned)M), block(NT);
    switch (vpt) {
#define H3B_RCASE(V) \
    case V: quant_convrot_kernel<V, NT, G, SWIGLU><<<grid, block, 0, s>>>(x, ldx, K, xq, xs); break;
        H3B_RCASE(1) H3B_RCASE(2) H3B_RCASE(3) H3B_RCASE(4) H3B_RCASE(5) H3B_RCASE(6) H3B_RCASE(7) H3B_RCASE(8)
        H3B_RCASE(10) H3B_RCASE(12) H3B_RCASE(14) H3B_RCASE(16)
#undef H3B_RCASE
        default: break;
    }
}

template <int NT, Act ACT, bool GATHER = false>
static void launch_quant(int vpt, const uint16_t* x, int64_t ldx, int64_t M, int K, int8_t* xq, float* xs,
                         cudaStream_t s, GatherRows g = GatherRows{}) {
    dim3 grid((unsigned)M), block(NT);
    switch (vpt) {
#define H3B_QCASE(V) \
    case V: quant_rowwise_kernel<V, NT, ACT, GATHER><<<grid, block, 0, s>>>(x, ldx, K, xq, xs, g); break;
        H3B_QCASE(1) H3B_QCASE(2) H3B_QCASE(3) H3B_QCASE(4) H3B_QCASE(5) H3B_QCASE(6) H3B_QCASE(7) H3B_QCASE(8)
        H3B_QCASE(10) H3B_QCASE(12) H3B_QCASE(14) H3B_QCASE(16)
#undef H3B_QCASE
        default: break;
    }
}

static int pick_vpt(int need) {
    static const int opts[] = {1, 2, 3, 4, 5, 6, 7, 8, 10, 12, 14, 16};
    for (int o : opts)
        if (o >= need) return o;
    return -1;
}

template <Act ACT>
static int quant_impl(const void* x, int64_t ldx, int64_t M, int64_t K, int8_t* xq, float* xs, cudaStream_t s,
                      const char* who) {
    H3B_REQUIRE(x && xq && xs, "%s: NULL pointer", who);
    H3B_REQUIRE(M >= 0 && K > 0 && K % 8 == 0 && K <= 32768, "%s: K=%lld must be a positive multiple of 8 <= 32768", who,
                (long long)K);
    H3B_REQUIRE(ldx >= K && ldx % 8 == 0 && aligned(x, 16),
                "%s: x must be 16-byte aligned with ldx %% 8 == 0 (ldx=%lld)", who, (long long)ldx);
    H3B_REQUIRE(aligned(xq, 8), "%s: xq must be 8-byte aligned", who);
    H3B_REQUIRE(M < (1ll << 31), "%s: M too large", who);
    if (M == 0) return H3B_OK;
    const int nvec = (int)(K / 8);
    // 128 threads per row up to 8 vectors each (K <= 8192); longer rows take 256
    // threads (K = 13824: 0.92 vs 0.79 of the measured HBM bandwidth, fewer
    // registers per thread and more rows resident)
    int vpt = pick_vpt((nvec + 127) / 128);
    if (vpt > 8) vpt = -1;
    if (vpt > 0) {
        launch_quant<128, ACT>(vpt, static_cast<const uint16_t*>(x), ldx, M, (int)K, xq, xs, s);
    } else {
        vpt = pick_vpt((nvec + 255) / 256);
        launch_quant<256, ACT>(vpt, static_cast<const uint16_t*>(x), ldx, M, (int)K, xq, xs, s);
    }
    H3B_CUDA_TRY(cudaGetLastError());
    return H3B_OK;
}

int quant_rowwise(const void* x, int64_t ldx, int64_t M, int64_t K, int8_t* xq, float* xs, cudaStream_t s) {
    return quant_impl<Act::kNone>(x, ldx, M, K, xq, xs, s, "h3b_quant_rowwise");
}

template <bool SWIGLU>
static int quant_convrot(const void* x, int64_t ldx, int64_t M, int64_t K, int64_t group, int8_t* xq, float* xs,
                         cudaStream_t s, const char* who) {
    H3B_REQUIRE(x && xq && xs, "%s: NULL pointer", who);
    H3B_REQUIRE(group == 64 || group == 256, "%s: group=%lld (64 or 256 supported)", who, (long long)group);
    H3B_REQUIRE(M >= 0 && M < (1ll << 31) && K > 0 && K % group == 0 && K <= 32768,
                "%s: K=%lld must be a positive multiple of the group (%lld), <= 32768", who, (long long)K,
                (long long)group);
    const int64_t row = SWIGLU ? 2 * K : K;
    H3B_REQUIRE(ldx >= row && ldx % 8 == 0 && aligned(x, 16),
                "%s: x must be 16-byte aligned with ldx >= %lld and ldx %% 8 == 0", who, (long long)row);
    H3B_REQUIRE(aligned(xq, 8), "%s: xq must be 8-byte aligned", who);
    if (M == 0) return H3B_OK;
    const int nvec = (int)(K / 8);
    const uint16_t* xp = static_cast<const uint16_t*>(x);
    int vpt = pick_vpt((nvec + 127) / 128);
    if (vpt > 0) {
        if (group == 256) launch_convrot<128, 256, SWIGLU>(vpt, xp, ldx, M, (int)K, xq, xs, s);
        else launch_convrot<128, 64, SWIGLU>(vpt, xp, ldx, M, (int)K, xq, xs, s);
    } else {
        vpt = pick_vpt((nvec + 255) / 256);
        if (group == 256) launch_convrot<256, 256, SWIGLU>(vpt, xp, ldx, M, (int)K, xq, xs, s);
        else launch_convrot<256, 64, SWIGLU>(vpt, xp, ldx, M, (int)K, xq, xs, s);
    }
    H3B_CUDA_TRY(cudaGetLastError());
    return H3B_OK;
}

static int gather_quant(const void* const* src, int64_t src_ld, int64_t row_start, int64_t M, int64_t chunk_bytes,
                        int world, int8_t* xq, float* xs, cudaStream_t s) {
    const char* who = "h3b_a2a_inv_quant";
    H3B_REQUIRE(src && xq && xs && world >= 1 && world <= kMaxGatherRanks, "%s: bad arguments (world=%d)", who, world);
    H3B_REQUIRE(chunk_bytes > 0 && chunk_bytes % 16 == 0 && src_ld >= chunk_bytes && src_ld % 16 == 0,
                "%s: chunk %lld / src_ld %lld bytes must be multiples of 16", who, (long long)chunk_bytes,
                (long long)src_ld);
    const int64_t K = world * chunk_bytes / 2;
    H3B_REQUIRE(K <= 32768 && M >= 0 && M < (1ll << 31) && row_start >= 0, "%s: K=%lld / M=%lld out of range", who,
                (long long)K, (long long)M);
    H3B_REQUIRE(aligned(xq, 8), "%s: xq must be 8-byte aligned", who);
    GatherRows g{};
    for (int j = 0; j < world; ++j) {
        H3B_REQUIRE(src[j] && aligned(src[j], 16), "%s: src[%d] NULL or not 16-byte aligned", who, j);
        g.src[j] = static_cast<const uint4*>(src[j]);
    }
    g.row0 = row_start;
    g.ldv = src_ld / 16;
    g.cv = (int)(chunk_bytes / 16);
    if (M == 0) return H3B_OK;
    const int nvec = (int)(K / 8);
    int vpt = pick_vpt((nvec + 127) / 128);
    if (vpt > 0) {
        launch_quant<128, Act::kNone, true>(vpt, nullptr, 0, M, (int)K, xq, xs, s, g);
    } else {
        vpt = pick_vpt((nvec + 255) / 256);
        launch_quant<256, Act::kNone, true>(vpt, nullptr, 0, M, (int)K, xq, xs, s, g);
    }
    H3B_CUDA_TRY(cudaGetLastError());
    return H3B_OK;
}

static int gelu_tanh(const void* x, void* y, int64_t n, cudaStream_t s) {
    H3B_REQUIRE(x && y, "h3b_gelu_tanh: NULL pointer");
    H3B_REQUIRE(n >= 0 && n % 2 == 0, "h3b_gelu_tanh: n=%lld must be even", (long long)n);
    H3B_REQUIRE(aligned(x, 16) && aligned(y, 16), "h3b_gelu_tanh: x and y must be 16-byte aligned");
    if (n == 0) return H3B_OK;
    const int64_t nvec = n / 8;
    const int tail_pairs = (int)((n % 8) / 2);
    const int64_t sms = num_sms_here();
    const uint16_t* xb = static_cast<const uint16_t*>(x);
    uint16_t* yb = static_cast<uint16_t*>(y);
    if (int rc = gelu_table_ready(s)) return rc;
    DeviceStatus ds;
    if (int rc = device_status(&ds)) return rc;
    const int64_t lut_want = cdiv(nvec, kLutThreads);
    const unsigned lut_grid = (unsigned)(lut_want < 1 ? 1 : (lut_want < sms ? lut_want : sms));
    gelu_lut_kernel<<<lut_grid, kLutThreads, kTableBytes, s>>>(
        reinterpret_cast<const uint4*>(x), reinterpret_cast<uint4*>(y), nvec,
        reinterpret_cast<const uint32_t*>(xb + nvec * 8), reinterpret_cast<uint32_t*>(yb + nvec * 8), tail_pairs,
        ds.word);
    H3B_CUDA_TRY(cudaGetLastError());
    return H3B_OK;
}

}  // namespace h3b

extern "C" int h3b_gelu_tanh(const void* x, void* y, int64_t n, void* stream) {
    return h3b::gelu_tanh(x, y, n, static_cast<cudaStream_t>(stream));
}

extern "C" int h3b_quant_rowwise(const void* x, int64_t ldx, int64_t M, int64_t K, int8_t* xq, float* xs,
                                 void* stream) {
    return h3b::quant_rowwise(x, ldx, M, K, xq, xs, static_cast<cudaStream_t>(stream));
}

extern "C" int h3b_gelu_quant(const void* u, int64_t ldu, int64_t M, int64_t K, int8_t* xq, float* xs,
                              void* stream) {
    using namespace h3b;
    const char* who = "h3b_gelu_quant";
    H3B_REQUIRE(u && xq && xs, "%s: NULL pointer", who);
    H3B_REQUIRE(M >= 0 && M < (1ll << 31) && K > 0 && K % 8 == 0 && K <= 32768,
                "%s: K=%lld must be a positive multiple of 8 <= 32768", who, (long long)K);
    H3B_REQUIRE(ldu >= K && ldu % 8 == 0 && aligned(u, 16),
                "%s: u must be 16-byte aligned with ldu %% 8 == 0 (ldu=%lld)", who, (long long)ldu);
    H3B_REQUIRE(aligned(xq, 8), "%s: xq must be 8-byte aligned", who);
    if (M == 0) return H3B_OK;
    return gelu_quant_lut(static_cast<const uint16_t*>(u), ldu, M, (int)K, xq, xs, static_cast<cudaStream_t>(stream));
}

extern "C" int h3b_a2a_inv_quant(const void* const* src, int64_t src_ld, int64_t row_start, int64_t M,
                                 int64_t chunk_bytes, int world, int8_t* xq, float* xs, void* stream) {
    return h3b::gather_quant(src, src_ld, row_start, M, chunk_bytes, world, xq, xs, static_cast<cudaStream_t>(stream));
}

extern "C" int h3b_quant_rowwise_convrot(const void* x, int64_t ldx, int64_t M, int64_t K, int64_t group, int8_t* xq,
                                         float* xs, void* stream) {
    return h3b::quant_convrot<false>(x, ldx, M, K, group, xq, xs, static_cast<cudaStream_t>(stream),
                                     "h3b_quant_rowwise_convrot");
}

extern "C" int h3b_swiglu_quant_convrot(const void* x, int64_t ldx, int64_t M, int64_t K, int64_t group, int8_t* xq,
                                        float* xs, void* stream) {
    return h3b::quant_convrot<true>(x, ldx, M, K, group, xq, xs, static_cast<cudaStream_t>(stream),
                                    "h3b_swiglu_quant_convrot");
}
