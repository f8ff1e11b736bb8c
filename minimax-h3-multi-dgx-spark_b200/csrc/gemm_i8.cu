// a2: INT8 x INT8 -> INT32 GEMM on 5th-generation tensor cores (tcgen05,
// kind::i8) with the fp32 dequant (+bias) epilogue fused, for sm_100a.
//
//   out[m,n] = bf16((float(acc[m,n]) * xs[m]) * ws[n] [+ float(bias[n])])
//   acc[m,n] = sum_k xq[m,k] * w[n,k]          (both operands K-contiguous)
//
// Design (one CTA per SM, persistent):
//   warp 0      TMA producer: 128x128-byte A tiles and 256x128-byte B tiles,
//               128B-swizzled, into a STAGES-deep shared-memory ring
//               (no cluster multicast: each CTA loads its own tiles).
//   warp 1      allocates 512 TMEM columns and issues the MMAs from one
//               thread: 4 x tcgen05.mma M=128 N=256 K=32 per stage into one
//               of two 256-column int32 accumulators; tcgen05.commit frees the
//               stage and, after the last k-block, hands the accumulator over.
//   warps 2..    epilogue (4 warps; 8 in the plain 2-CTA variant, two per lane
//               quarter): tcgen05.ld 32 columns at a time (warp w reads TMEM
//               lanes 32*(w%4)..+31 = tile rows), dequantise with separate
//               IEEE multiplies (no FMA contraction: the reference rounds
//               after each product), round once to bf16, store; then release
//               the accumulator so the MMA warp can start the tile after next
//               while this one drains.
// Tiles are visited in the reference's grouped-M order (int8_gemm_triton.py:37-45,
// GROUP_M = 8 there; 16 tile rows per group here, chosen by measurement) so
// CTAs running at the same time share A and B rows in L2.  Every mbarrier wait
// is bounded; on expiry the kernel records H3B_STATUS_MBAR_TIMEOUT, stops
// issuing work, drains its own TMA loads and MMAs (again bounded), frees TMEM
// and returns.
#include <mutex>
#include <cuda.h>
#include <stdlib.h>

#include "common.cuh"
#include "quant_common.cuh"  // gelu2

namespace h3b {
namespace gemm {

constexpr int BM = 128;                  // tile rows (TMEM lanes)
constexpr int BN = 256;                  // tile columns (TMEM columns per accumulator)
constexpr int BK = 128;                  // k-block in bytes = one 128B swizzle row
constexpr int UMMA_K = 32;               // K per kind::i8 instruction
constexpr int STAGES = 4;
constexpr int NUM_ACC = 2;
constexpr int TMEM_COLS = NUM_ACC * BN;  // 512: the whole TMEM of the SM
constexpr int A_BYTES = BM * BK;
constexpr int B_BYTES = BN * BK;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int GROUP_M = 16;  // tile rows per group of the grouped-M raster
constexpr int kThreads = 192;
constexpr int kEpiWarps = 4;
constexpr uint64_t kTimeoutNs = 10ull * 1000 * 1000 * 1000;
constexpr int kSmemBytes = STAGES * STAGE_BYTES + 1024 /*alignment slack*/ + 256 /*barriers*/;

// Instruction descriptor: D s32 (bits 4-5 = 2), A s8 (7-9 = 1), B s8 (10-12 = 1),
// both K-major (bits 15/16 = 0), N >> 3 at bits 17-22, M >> 4 at bits 24-28.
constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                            ((uint32_t)(BM >> 4) << 24);

constexpr int kMaxScatterSegs = 3;   // q, k, v
constexpr int kMaxScatterWorld = 8;

// Scatter epilogue: the GEMM fused with the Ulysses forward exchange.  Output
// column n lies in segment t = n / seg (q, k, v), head h = (n % seg) / head_dim,
// which rank j = h / hp owns; it is stored into rank j's receive buffer
// dst[t * world + j] (a peer's memory for j != this rank) at row row_start + m
// and column (h - j*hp)*head_dim + n % head_dim, receive rows being
// hp*head_dim elements wide -- the layout the exchange delivers.
struct Scatter {
    uint16_t* dst[kMaxScatterSegs * kMaxScatterWorld];
    int64_t row_start;
    int seg, head_dim, hp, world;
    // Optional per-head RMSNorm of the first norm_segs segments (the q and k
    // norms of the attention): each 128-column head of those segments becomes
    // rbf16(w_t * (rstd * y)), w_t = norm_w + t * 128, before it is stored.
    const uint16_t* norm_w;
    int norm_segs;
    float norm_eps;
};

struct Args {
    const float* xs;
    const float* ws;
    const uint16_t* bias;
    void* out;
    int M, N, K;
    int* status;
    int tile_n;  // 2-CTA kernel: output tile width (multiple of 32, <= 256)
    int group_m; // tile rows per group of the grouped-M raster
    Scatter sc;  // scatter epilogue only
    int act;     // bf16 output: 1 = GELU(tanh) applied to each rounded output value
};

// ---------------------------------------------------------------------------
// PTX wrappers

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with the given parity to complete.  Returns false
// if the kernel is aborting (another role timed out) or this wait timed out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* status,
                                          uint64_t limit_ns = kTimeoutNs) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t n = 1;; ++n) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((n & 127u) == 0) {
            if (*abort_flag) return false;
            if (globaltimer_ns() - t0 > limit_ns) {
                *abort_flag = 1;
                report(status, H3B_STATUS_MBAR_TIMEOUT);
                return false;
            }
        }
    }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor, K-major, 128-byte swizzle: start address
// >> 4 (bits 0-13), leading byte offset 16 B (unused with swizzle), stride
// byte offset 1024 B = 8 rows x 128 B (bits 32-45), descriptor version 1
// (bit 46), layout SWIZZLE_128B = 2 (bits 61-63).  Stepping K by 32 bytes
// inside the 128-byte swizzle row advances the start address; the hardware
// applies the XOR swizzle to the final address, matching TMA's layout.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tile_coords(int tile, int m_tiles, int n_tiles, int group_m, int& mb, int& nb) {
    const int in_group = group_m * n_tiles;
    const int group = tile / in_group;
    const int first_m = group * group_m;
    const int gsize = min(m_tiles - first_m, group_m);
    const int r = tile % in_group;
    mb = first_m + r % gsize;
    nb = r / gsize;
}

// bf16((float(acc) * xs) * ws[n] [+ bias[n]]) of 8 columns cb .. cb+7 of one
// row (int32 sums r[0..7]) with separate IEEE products, packed in pairs.
__device__ __forceinline__ uint4 dequant8(const Args& args, const uint32_t* r, int cb, float xs) {
    const float4 w0 = *reinterpret_cast<const float4*>(args.ws + cb);
    const float4 w1 = *reinterpret_cast<const float4*>(args.ws + cb + 4);
    const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    float bv[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (args.bias) {
        const uint4 b = *reinterpret_cast<const uint4*>(args.bias + cb);
        const uint32_t bu[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            bv[2 * e] = bf16_lo(bu[e]);
            bv[2 * e + 1] = bf16_hi(bu[e]);
        }
    }
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        float v0 = __fmul_rn(__fmul_rn(__int2float_rn((int)r[2 * e]), xs), wv[2 * e]);
        float v1 = __fmul_rn(__fmul_rn(__int2float_rn((int)r[2 * e + 1]), xs), wv[2 * e + 1]);
        if (args.bias) {
            v0 = __fadd_rn(v0, bv[2 * e]);
            v1 = __fadd_rn(v1, bv[2 * e + 1]);
        }
        o[e] = pack_bf16x2(v0, v1);
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

// Dequantise one 32-column chunk of one tile row (registers r) and store it:
// out[row, col0 .. col0+31] = bf16((float(acc) * xs) * ws[n] [+ bias[n]]), or
// the raw int32 sums.  N % 8 == 0, so every 8-column group is either fully
// inside or fully outside the matrix.
template <bool OUT_I32>
__device__ __forceinline__ void store_chunk(const Args& args, const uint32_t (&r)[32], int row, int col0, float xs) {
    const int N = args.N;
    if constexpr (OUT_I32) {
        int4* dst = reinterpret_cast<int4*>(static_cast<int32_t*>(args.out) + (int64_t)row * N + col0);
#pragma unroll
        for (int g = 0; g < 8; ++g)
            if (col0 + 4 * g < N) dst[g] = make_int4((int)r[4 * g], (int)r[4 * g + 1], (int)r[4 * g + 2], (int)r[4 * g + 3]);
    } else {
        uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(args.out) + (int64_t)row * N + col0);
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            const int cb = col0 + 8 * g;
            if (cb >= N) break;
            uint4 y = dequant8(args, r + 8 * g, cb, xs);
            if (args.act) y = make_uint4(gelu2(y.x), gelu2(y.y), gelu2(y.z), gelu2(y.w));
            dst[g] = y;
        }
    }
}

// Scatter epilogue of one 64-column unit of the 32 tile rows row0 .. row0+31
// held by this warp (lane = row): dequantise into the warp's 4 KB staging
// area (row-major 32 x 128 B, 16-byte pieces XOR-swizzled by row so that both
// the row-wise writes and the piece-wise reads are conflict-free), then store
// it with 8 lanes per row, so every store instruction writes four whole
// 128-byte lines -- full NVLink writes when the destination is a peer.
// Requires seg % head_dim == 0 and head_dim % 64 == 0 (a unit never straddles
// a head, so its destination is warp-uniform).
__device__ __forceinline__ void store_stage(const Args& args, const uint4* stage, int row0, int col0, int lane);

__device__ __forceinline__ void scatter_unit(const Args& args, uint4* stage, uint32_t t_col, int row0, int col0,
                                            float xs, int lane) {
    uint32_t r[32];
    tmem_ld32(t_col, r);
#pragma unroll
    for (int g = 0; g < 4; ++g) stage[lane * 8 + (g ^ (lane & 7))] = dequant8(args, r + 8 * g, col0 + 8 * g, xs);
    tmem_ld32(t_col + 32u, r);
#pragma unroll
    for (int g = 0; g < 4; ++g)
        stage[lane * 8 + ((g + 4) ^ (lane & 7))] = dequant8(args, r + 8 * g, col0 + 32 + 8 * g, xs);
    __syncwarp();
    store_stage(args, stage, row0, col0, lane);
}

// The staged 32 rows x 64 columns (columns col0 ..) to the owning rank's
// receive buffer, 8 lanes per row.
__device__ __forceinline__ void store_stage(const Args& args, const uint4* stage, int row0, int col0, int lane) {
    const Scatter& sc = args.sc;
    const int t = col0 / sc.seg, within = col0 - t * sc.seg;
    const int h = within / sc.head_dim, j = h / sc.hp;
    const int64_t dld = (int64_t)sc.hp * sc.head_dim;
    uint16_t* dbase = sc.dst[t * sc.world + j] + (int64_t)(h - j * sc.hp) * sc.head_dim + (within % sc.head_dim);
#pragma unroll
    for (int p = 0; p < 8; ++p) {
        const int e = p * 32 + lane, rr = e >> 3, cc = e & 7;
        const uint4 v = stage[rr * 8 + (cc ^ (rr & 7))];
        const int grow = row0 + rr;
        if (grow < args.M) *reinterpret_cast<uint4*>(dbase + (sc.row_start + grow) * dld + cc * 8) = v;
    }
    __syncwarp();
}

// Scatter epilogue of one 128-column head with its RMSNorm (q / k norm): the
// lane's row of the head is dequantised to bf16 (the projection's output),
// its sum of squares is formed in the order PyTorch's F.rms_norm uses for a
// 128-wide row (32 partial sums of 4 consecutive elements, each an FMA chain
// from 0, then the shuffle-down tree 16, 8, 4, 2, 1 over the partials; the
// other warps of that reduction contribute exact zeros), rstd =
// rsqrtf(sum / 128 + eps), and each element becomes rbf16(w * (rstd * y)).
// The normalised head is stored as two staged 64-column halves.
__device__ __forceinline__ void scatter_head_norm(const Args& args, uint4* stage, uint32_t t_col, int row0, int col0,
                                                 float xs, int lane, const uint16_t* __restrict__ w) {
    uint32_t hw[64];  // the head's 128 bf16 values, packed in pairs
    float part[16];   // partial sums after the tree's first level (16)
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(t_col + 32u * c, r);
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            const uint4 v = dequant8(args, r + 8 * g, col0 + 32 * c + 8 * g, xs);
            hw[16 * c + 4 * g + 0] = v.x;
            hw[16 * c + 4 * g + 1] = v.y;
            hw[16 * c + 4 * g + 2] = v.z;
            hw[16 * c + 4 * g + 3] = v.w;
        }
        // partials of virtual threads 8c .. 8c+7 (elements 4vt .. 4vt+3 = words 2vt, 2vt+1)
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int vt = 8 * c + k;
            float acc = 0.0f;
            acc = __fmaf_rn(bf16_lo(hw[2 * vt]), bf16_lo(hw[2 * vt]), acc);
            acc = __fmaf_rn(bf16_hi(hw[2 * vt]), bf16_hi(hw[2 * vt]), acc);
            acc = __fmaf_rn(bf16_lo(hw[2 * vt + 1]), bf16_lo(hw[2 * vt + 1]), acc);
            acc = __fmaf_rn(bf16_hi(hw[2 * vt + 1]), bf16_hi(hw[2 * vt + 1]), acc);
            if (c < 2) part[vt] = acc;                          // vt < 16
            else part[vt - 16] = __fadd_rn(part[vt - 16], acc);  // tree level 16
        }
    }
#pragma unroll
    for (int off = 8; off >= 1; off >>= 1)
#pragma unroll
        for (int vt = 0; vt < off; ++vt) part[vt] = __fadd_rn(part[vt], part[vt + off]);
    const float tot = __fadd_rn(__fadd_rn(part[0], 0.0f), __fadd_rn(0.0f, 0.0f));
    // tot / 128: a multiply by 2^-7 rounds the same exact quotient as the division
    const float rstd = rsqrtf(__fadd_rn(__fmul_rn(tot, 0.0078125f), args.sc.norm_eps));
    const uint4* wv = reinterpret_cast<const uint4*>(w);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
#pragma unroll
        for (int g = 0; g < 8; ++g) {
            const uint4 w4 = wv[8 * half + g];
            const uint32_t ww[4] = {w4.x, w4.y, w4.z, w4.w};
            uint32_t o[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const uint32_t x = hw[32 * half + 4 * g + e];
                o[e] = pack_bf16x2(__fmul_rn(bf16_lo(ww[e]), __fmul_rn(rstd, bf16_lo(x))),
                                   __fmul_rn(bf16_hi(ww[e]), __fmul_rn(rstd, bf16_hi(x))));
            }
            stage[lane * 8 + (g ^ (lane & 7))] = make_uint4(o[0], o[1], o[2], o[3]);
        }
        __syncwarp();
        store_stage(args, stage, row0, col0 + 64 * half, lane);
    }
}

// ---------------------------------------------------------------------------

template <bool OUT_I32>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_i8_kernel(
const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, Args args) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* sA = base;
    uint8_t* sB = base + STAGES * A_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * B_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + NUM_ACC;
    uint64_t* drain = tempty + NUM_ACC;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < NUM_ACC; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], kEpiWarps);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmA) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmB) : "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int M = args.M, N = args.N, K = args.K;
    const int m_tiles = (M + BM - 1) / BM, n_tiles = (N + BN - 1) / BN;
    const int num_tiles = m_tiles * n_tiles;
    const int kblocks = K / BK;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer
            int stage = 0;
            uint32_t phase = 0;
            int armed = 0;  // loads issued (bounded drain below needs the last STAGES)
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
                int mb, nb;
                tile_coords(tile, m_tiles, n_tiles, args.group_m, mb, nb);
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, args.status)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(&full[stage], STAGE_BYTES);
                    tma_load_2d(sA + stage * A_BYTES, &tmA, &full[stage], kb * BK, mb * BM);
                    tma_load_2d(sB + stage * B_BYTES, &tmB, &full[stage], kb * BK, nb * BN);
                    ++armed;
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (!ok) {
                // Let the loads this thread issued land before the CTA exits:
                // walk back over the last (up to STAGES) armed stages.
                int s = stage;
                uint32_t p = phase;
                for (int i = 0; i < STAGES && i < armed; ++i) {
                    if (--s < 0) {
                        s = STAGES - 1;
                        p ^= 1u;
                    }
                    volatile int no_abort = 0;
                    mbar_wait(&full[s], p, &no_abort, nullptr, 100ull * 1000 * 1000);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer
            int stage = 0;
            uint32_t phase = 0;
            int t = 0;
            bool ok = true;
            bool issued = false;
            for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x, ++t) {
                const int acc = t & 1;
                const uint32_t acc_phase = (uint32_t)(t >> 1) & 1u;
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, args.status)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&full[stage], phase, abort_flag, args.status)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sA + stage * A_BYTES);
                    const uint32_t b0 = smem_u32(sB + stage * B_BYTES);
#pragma unroll
                    for (int kk = 0; kk < BK / UMMA_K; ++kk)
                        umma_i8(d_tmem, smem_desc(a0 + kk * UMMA_K), smem_desc(b0 + kk * UMMA_K), (kb | kk) != 0);
                    issued = true;
                    umma_commit(&empty[stage]);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (ok) umma_commit(&tfull[acc]);
            }
            if (!ok && issued) {
                // Wait (bounded) until every MMA this thread issued has finished.
                umma_commit(drain);
                volatile int no_abort = 0;
                mbar_wait(drain, 0, &no_abort, nullptr, 100ull * 1000 * 1000);
            }
        }
    } else {
        // ---------------- epilogue warps 2..5
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        int t = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++t) {
            int mb, nb;
            tile_coords(tile, m_tiles, n_tiles, args.group_m, mb, nb);
            const int acc = t & 1;
            const uint32_t acc_phase = (uint32_t)(t >> 1) & 1u;
            if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, args.status)) break;
            tc_fence_after();
            const int row = mb * BM + q * 32 + lane;
            const bool row_ok = row < M;
            float xs = 0.0f;
            if constexpr (!OUT_I32) xs = row_ok ? args.xs[row] : 0.0f;
            const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                const int col0 = nb * BN + c * 32;
                if (col0 >= N) break;  // warp-uniform
                uint32_t r[32];
                tmem_ld32(t_row + (uint32_t)(c * 32), r);
                if (row_ok) store_chunk<OUT_I32>(args, r, row, col0, xs);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[acc]);
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                     : "memory");
}

// ---------------------------------------------------------------------------
// 2-CTA variant (cluster of 2, tcgen05 cta_group::2).  A pair of CTAs owns a
// 256 x tile_n output tile (tile_n = 32..256, chosen per launch): CTA rank c
// loads rows [c*128, c*128+128) of the tile's A rows AND rows
// [c*tile_n/2, (c+1)*tile_n/2) of its B rows (plain TMA into its
// own shared memory; the .cta_group::2 load form lets both CTAs signal the
// leader's stage barrier).  The leader (rank 0) issues
// tcgen05.mma.cta_group::2 M=256 N=tile_n K=32, which reads A and B halves from
// both CTAs and accumulates rows c*128.. into CTA c's TMEM.  Per SM this moves
// 32 KiB per 128-byte k-block instead of 48 KiB, cutting L2->SM traffic by a
// third.  Commits multicast to both CTAs' barriers; both CTAs' epilogue warps
// release an accumulator on the leader's barrier.  No TMA multicast is used.
namespace pair {

constexpr int BM = 128;  // A rows per CTA; the pair tile has 256
constexpr int TILE_M = 256;
constexpr int MAX_TILE_N = 256;  // tile width is a launch parameter: 32..256, multiple of 32
constexpr int B_ROWS = 128;      // B rows per CTA at the widest tile
constexpr int STAGES = 6;
constexpr int A_BYTES = BM * BK;
constexpr int B_BYTES = B_ROWS * BK;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int kSmemBytes = STAGES * STAGE_BYTES + 1024 + 256;
// Epilogue warps.  The plain variant has two per TMEM lane quarter (warps w
// and w + 4 read the same 32 accumulator rows and take alternate 32-column
// chunks), so the dequantisation (and the GELU) of one accumulator runs on
// eight warps while the MMAs fill the other.  The scatter variant keeps one
// per quarter: its q/k-norm epilogue holds a whole 128-column head per thread
// (255 registers); at 320 threads, capped at 200 registers, it spilled and its
// launch was refused for resources.
template <bool SCATTER>
constexpr int epi_warps() { return SCATTER ? 4 : 8; }
template <bool SCATTER>
constexpr int threads() { return 64 + 32 * epi_warps<SCATTER>(); }  // TMA producer, MMA issuer, epilogue
constexpr int kStagingBytes = epi_warps<true>() * 32 * 128;  // scatter epilogue: 32 rows x 128 B per warp
constexpr int kSmemBytesScatter = kSmemBytes + kStagingBytes;
static_assert(kSmemBytesScatter <= 227 * 1024, "shared memory of the scatter variant above the 227 KB per CTA");
// instruction descriptor without its N field (bits 17-22 = N >> 3, set per launch)
constexpr uint32_t kIdescBase = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(TILE_M >> 4) << 24);

__device__ __forceinline__ uint32_t ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// address of the same shared variable in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint32_t mbar_cluster, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
        "[%2];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(mbar_cluster), "r"(c0), "r"(c1)
        : "memory");
}
__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// arrive (when the MMAs issued so far complete) on `bar` in both CTAs of the pair
__device__ __forceinline__ void umma_commit_both(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"((uint16_t)0x3)
        : "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

template <bool OUT_I32, bool SCATTER>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(threads<SCATTER>(), 1)
    gemm_i8_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, Args args) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* sA = base;
    uint8_t* sB = base + STAGES * A_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * B_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + NUM_ACC;
    uint64_t* drain = tempty + NUM_ACC;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = ctarank();
    const bool leader = rank == 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < NUM_ACC; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 2 * epi_warps<SCATTER>());
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmA) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmB) : "memory");
    }
    if (warp == 1) {
        // one warp with the same warp id in each CTA of the pair, same slot offset
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    cluster_sync();  // barrier inits and the TMEM allocation are visible to both CTAs
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int M = args.M, N = args.N, K = args.K;
    const int TILE_N = args.tile_n;
    const int b_rows = TILE_N / 2;  // B rows this CTA loads
    const uint32_t idesc = kIdescBase | ((uint32_t)(TILE_N >> 3) << 17);
    const uint32_t stage_tx = 2u * (uint32_t)(A_BYTES + b_rows * BK);
    const int m_tiles = (M + TILE_M - 1) / TILE_M, n_tiles = (N + TILE_N - 1) / TILE_N;
    const int num_tiles = m_tiles * n_tiles;
    const int kblocks = K / BK;
    const int pair_id = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer (both CTAs; the leader also arms the stage barrier)
            int stage = 0;
            uint32_t phase = 0;
            int armed = 0;
            bool ok = true;
            for (int tile = pair_id; ok && tile < num_tiles; tile += n_pairs) {
                int mb, nb;
                tile_coords(tile, m_tiles, n_tiles, args.group_m, mb, nb);
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, args.status)) {
                        ok = false;
                        break;
                    }
                    if (leader) mbar_expect_tx(&full[stage], stage_tx);
                    const uint32_t fb = mapa(smem_u32(&full[stage]), 0);
                    tma_load_2d(sA + stage * A_BYTES, &tmA, fb, kb * BK, mb * TILE_M + (int)rank * BM);
                    tma_load_2d(sB + stage * B_BYTES, &tmB, fb, kb * BK, nb * TILE_N + (int)rank * b_rows);
                    ++armed;
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (!ok) {
                if (leader) {
                    // the leader's stage barriers count both CTAs' bytes: wait (bounded)
                    // until the armed stages have landed
                    int s = stage;
                    uint32_t p = phase;
                    for (int i = 0; i < STAGES && i < armed; ++i) {
                        if (--s < 0) {
                            s = STAGES - 1;
                            p ^= 1u;
                        }
                        volatile int no_abort = 0;
                        mbar_wait(&full[s], p, &no_abort, nullptr, 100ull * 1000 * 1000);
                    }
                } else {
                    const uint64_t t0 = globaltimer_ns();  // let this CTA's loads in flight land
                    while (globaltimer_ns() - t0 < 2000000ull) __nanosleep(1000);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            // ---------------- MMA issuer (leader CTA only)
            int stage = 0;
            uint32_t phase = 0;
            int t = 0;
            bool ok = true;
            bool issued = false;
            for (int tile = pair_id; ok && tile < num_tiles; tile += n_pairs, ++t) {
                const int acc = t & 1;
                const uint32_t acc_phase = (uint32_t)(t >> 1) & 1u;
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, args.status)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(acc * MAX_TILE_N);
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&full[stage], phase, abort_flag, args.status)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sA + stage * A_BYTES);
                    const uint32_t b0 = smem_u32(sB + stage * B_BYTES);
#pragma unroll
                    for (int kk = 0; kk < BK / UMMA_K; ++kk)
                        umma_i8(d_tmem, smem_desc(a0 + kk * UMMA_K), smem_desc(b0 + kk * UMMA_K), idesc,
                                (kb | kk) != 0);
                    issued = true;
                    umma_commit_both(&empty[stage]);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (ok) umma_commit_both(&tfull[acc]);
            }
            if (!ok && issued) {
                umma_commit_both(drain);
                volatile int no_abort = 0;
                mbar_wait(drain, 0, &no_abort, nullptr, 100ull * 1000 * 1000);
            }
        }
    } else {
        // ---------------- epilogue warps 2 .. (both CTAs: rows rank*128 .. of the pair tile)
        const int q = warp & 3;                                        // TMEM lane quarter of this warp
        const int ew = warp - 2;                                       // epilogue warp index
        const int part = ew >> 2, nparts = epi_warps<SCATTER>() / 4;  // this warp's share of the columns
        int t = 0;
        for (int tile = pair_id; tile < num_tiles; tile += n_pairs, ++t) {
            int mb, nb;
            tile_coords(tile, m_tiles, n_tiles, args.group_m, mb, nb);
            const int acc = t & 1;
            const uint32_t acc_phase = (uint32_t)(t >> 1) & 1u;
            if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, args.status)) break;
            tc_fence_after();
            const int row = mb * TILE_M + (int)rank * BM + q * 32 + lane;
            const bool row_ok = row < M;
            float xs = 0.0f;
            if constexpr (!OUT_I32) xs = row_ok ? args.xs[row] : 0.0f;
            const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * MAX_TILE_N);
            if constexpr (SCATTER) {
                // 64-column units (TILE_N % 64 == 0 and N % 64 == 0 for this variant)
                uint4* stage = reinterpret_cast<uint4*>(base + STAGES * STAGE_BYTES + 256) + ew * (32 * 8);
                // items: 64-column units, or whole 128-column heads when normalised
                // (tile_n % 128 == 0 then); with two warps per lane quarter they
                // take alternate items
#pragma unroll 1
                for (int c = 0, item = 0; c < TILE_N / 64; ++item) {
                    const int col0 = nb * TILE_N + c * 64;
                    if (col0 >= N) break;  // warp-uniform
                    const int t = col0 / args.sc.seg;
                    const bool norm = t < args.sc.norm_segs;
                    if (item % nparts == part) {
                        if (norm)
                            scatter_head_norm(args, stage, t_row + (uint32_t)(c * 64), row - lane, col0, xs, lane,
                                              args.sc.norm_w + t * 128);
                        else
                            scatter_unit(args, stage, t_row + (uint32_t)(c * 64), row - lane, col0, xs, lane);
                    }
                    c += norm ? 2 : 1;
                }
            } else {
#pragma unroll 1
                for (int c = part; c < TILE_N / 32; c += nparts) {
                    const int col0 = nb * TILE_N + c * 32;
                    if (col0 >= N) break;  // warp-uniform
                    uint32_t r[32];
                    tmem_ld32(t_row + (uint32_t)(c * 32), r);
                    if (row_ok) store_chunk<OUT_I32>(args, r, row, col0, xs);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(mapa(smem_u32(&tempty[acc]), 0));
        }
    }

    tc_fence_before();
    cluster_sync();  // both CTAs are done with TMEM (every MMA was consumed by an epilogue)
    tc_fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                     : "memory");
}

}  // namespace pair

// ---------------------------------------------------------------------------
// Host side

typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiled encode_fn() {
    static PFN_encodeTiled fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_encodeTiled>(p);
    }
    return fn;
}

// 2-D int8 tensor [rows, K] (K contiguous) tiled as box_rows x 128 bytes, 128B swizzle.
static int make_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t K, uint32_t box_rows) {
    PFN_encodeTiled enc = encode_fn();
    if (!enc) return set_error(H3B_ERR_CUDA, "cuTensorMapEncodeTiled unavailable (driver too old?)");
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)K};
    cuuint32_t box[2] = {(cuuint32_t)BK, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(H3B_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return H3B_OK;
}

static int num_sms() {
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return 148;
    return sms;
}

// Tile rows per group of the grouped-M raster (the weights are streamed once
// per group): GROUP_M = 16, measured on the block's four shapes at M=128000
// 2-4% faster than 8 on each (the weights are streamed half as often) and
// faster than 32 (whose A slabs no longer stay in L2 for K=13824).
// H3B_GEMM_GROUP_M overrides it for tuning sweeps.
static int pick_group_m() {
    static int forced = -1;
    if (forced < 0) {
        const char* e = getenv("H3B_GEMM_GROUP_M");
        const int v = e ? atoi(e) : 0;
        forced = (v >= 1 && v <= 256) ? v : 0;
    }
    return forced ? forced : GROUP_M;
}

// Output tile width of the 2-CTA kernel.  The kernel is bound by the L2->SM
// feed (measured: throughput at width t scales as 1 / (8192/t + 32) bytes per
// clock per SM), so a tile's run time is proportional to the operand rows it
// streams per k-block, 256 (A) + t (B).  The chosen width minimises
// (rounds of pair tiles over the resident pairs) x (256 + t); ties go to the
// wider tile.  Wave quantisation picks 224 for config 0's 4096 x 5120; large M
// keeps 256.
static int pick_tile_n(int M, int N, int64_t pairs, int multiple = 32) {
    // H3B_GEMM_TILE_N (a multiple of 32 in 32..256) pins the width, for tuning sweeps
    static int forced = -1;
    if (forced < 0) {
        const char* e = getenv("H3B_GEMM_TILE_N");
        const int v = e ? atoi(e) : 0;
        forced = (v >= 32 && v <= 256 && v % 32 == 0) ? v : 0;
    }
    if (forced && forced % multiple == 0) return forced;
    static const int cands[] = {256, 224, 192, 160, 128};
    const int64_t m_tiles = (M + pair::TILE_M - 1) / pair::TILE_M;
    int best = 256;
    int64_t best_cost = -1;
    for (int t : cands) {
        if (t % multiple) continue;
        const int64_t tiles = m_tiles * ((N + t - 1) / t);
        const int64_t rounds = (tiles + pairs - 1) / pairs;
        const int64_t cost = rounds * (256 + t);
        if (best_cost < 0 || cost < best_cost) {
            best_cost = cost;
            best = t;
        }
    }
    return best;
}

// H3B_GEMM_SINGLE_CTA=1 selects the 1-CTA kernel for every shape (the 2-CTA
// kernel is the default when M > 128).
static bool force_single_cta() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("H3B_GEMM_SINGLE_CTA");
        v = (e && e[0] == '1') ? 1 : 0;
    }
    return v == 1;
}

// How many CTA pairs can be resident at once (a GPC may not pair every SM);
// queried once per device and kernel variant, SM count / 2 if the query fails.
template <bool OUT_I32, bool SCATTER>
static int max_pairs() {
    constexpr int kMaxDevices = 64;
    static int cache[kMaxDevices] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return num_sms() / 2;
    if (cache[dev] > 0) return cache[dev];
    int n = 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (num_sms() / 2), 1, 1);
    cfg.blockDim = dim3(pair::threads<SCATTER>(), 1, 1);
    cfg.dynamicSmemBytes = SCATTER ? pair::kSmemBytesScatter : pair::kSmemBytes;
    if (cudaOccupancyMaxActiveClusters(&n, (void*)pair::gemm_i8_pair_kernel<OUT_I32, SCATTER>, &cfg) != cudaSuccess ||
        n <= 0) {
        cudaGetLastError();
        n = num_sms() / 2;
    }
    cache[dev] = n;
    return n;
}

static int check_device() {
    int dev = 0, major = 0;
    H3B_CUDA_TRY(cudaGetDevice(&dev));
    H3B_CUDA_TRY(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
    if (major != 10) return set_error(H3B_ERR_UNSUPPORTED, "libh3b GEMM needs an sm_100 GPU (found compute %d.x)", major);
    return H3B_OK;
}

template <bool OUT_I32, bool SCATTER = false>
static int launch(const int8_t* xq, const int8_t* w, Args a, cudaStream_t s) {
    H3B_REQUIRE(xq && w && (SCATTER || a.out), "h3b GEMM: NULL pointer");
    H3B_REQUIRE(a.M >= 0 && a.N > 0 && a.K > 0, "h3b GEMM: bad shape M=%d N=%d K=%d", a.M, a.N, a.K);
    H3B_REQUIRE(a.K % BK == 0, "h3b GEMM: K=%d must be a multiple of %d", a.K, BK);
    H3B_REQUIRE(a.N % 8 == 0, "h3b GEMM: N=%d must be a multiple of 8", a.N);
    H3B_REQUIRE(aligned(xq, 16) && aligned(w, 16) && (SCATTER || aligned(a.out, 16)),
                "h3b GEMM: operands must be 16-byte aligned");
    if (!OUT_I32) {
        H3B_REQUIRE(a.xs && a.ws && aligned(a.ws, 16), "h3b GEMM: xs/ws NULL or ws not 16-byte aligned");
        H3B_REQUIRE(!a.bias || aligned(a.bias, 16), "h3b GEMM: bias must be 16-byte aligned");
    }
    if (a.M == 0) return H3B_OK;
    a.group_m = pick_group_m();
    if (int rc = check_device()) return rc;
    CUtensorMap tmA, tmB;
    if (int rc = make_map(&tmA, xq, a.M, a.K, BM)) return rc;
    if (int rc = make_map(&tmB, w, a.N, a.K, BN)) return rc;
    DeviceStatus ds;
    if (int rc = device_status(&ds)) return rc;
    a.status = ds.word;
    if (SCATTER || (a.M > BM && !force_single_cta())) {
        // 2-CTA pairs: each CTA loads tile_n / 2 rows of B (the scatter epilogue
        // exists in this kernel only; rows past M are masked)
        constexpr int smem = SCATTER ? pair::kSmemBytesScatter : pair::kSmemBytes;
        H3B_CUDA_TRY(cudaFuncSetAttribute(pair::gemm_i8_pair_kernel<OUT_I32, SCATTER>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        const int64_t pairs_max = max_pairs<OUT_I32, SCATTER>();
        a.tile_n = pick_tile_n(a.M, a.N, pairs_max, !SCATTER ? 32 : (a.sc.norm_segs > 0 ? 128 : 64));
        if (int rc = make_map(&tmB, w, a.N, a.K, (uint32_t)(a.tile_n / 2))) return rc;
        const int64_t tiles = (int64_t)((a.M + pair::TILE_M - 1) / pair::TILE_M) * ((a.N + a.tile_n - 1) / a.tile_n);
        const int pairs = (int)(tiles < pairs_max ? tiles : pairs_max);
        pair::gemm_i8_pair_kernel<OUT_I32, SCATTER><<<2 * pairs, pair::threads<SCATTER>(), smem, s>>>(tmA, tmB, a);
    } else {
        H3B_CUDA_TRY(cudaFuncSetAttribute(gemm_i8_kernel<OUT_I32>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
        const int64_t tiles = (int64_t)((a.M + BM - 1) / BM) * ((a.N + BN - 1) / BN);
        const int grid = (int)(tiles < num_sms() ? tiles : num_sms());
        gemm_i8_kernel<OUT_I32><<<grid, kThreads, kSmemBytes, s>>>(tmA, tmB, a);
    }
    H3B_CUDA_TRY(cudaGetLastError());
    return H3B_OK;
}

}  // namespace gemm

int quant_rowwise(const void* x, int64_t ldx, int64_t M, int64_t K, int8_t* xq, float* xs, cudaStream_t s);

}  // namespace h3b

using namespace h3b;

static bool fits_int(int64_t v) { return v >= 0 && v < (1ll << 31); }

extern "C" int h3b_int8_mm_scaled(const int8_t* xq, const int8_t* w, const float* xs, const float* ws,
                                  const void* bias, void* out, int64_t M, int64_t N, int64_t K, void* stream) {
    H3B_REQUIRE(fits_int(M) && fits_int(N) && fits_int(K), "h3b_int8_mm_scaled: shape out of range");
    gemm::Args a{xs, ws, static_cast<const uint16_t*>(bias), out, (int)M, (int)N, (int)K, nullptr};
    return gemm::launch<false>(xq, w, a, static_cast<cudaStream_t>(stream));
}

extern "C" int h3b_int8_mm_scaled_gelu(const int8_t* xq, const int8_t* w, const float* xs, const float* ws,
                                       const void* bias, void* out, int64_t M, int64_t N, int64_t K, void* stream) {
    H3B_REQUIRE(fits_int(M) && fits_int(N) && fits_int(K), "h3b_int8_mm_scaled_gelu: shape out of range");
    gemm::Args a{xs, ws, static_cast<const uint16_t*>(bias), out, (int)M, (int)N, (int)K, nullptr};
    a.act = 1;
    return gemm::launch<false>(xq, w, a, static_cast<cudaStream_t>(stream));
}

extern "C" int h3b_int8_mm_i32(const int8_t* xq, const int8_t* w, int32_t* acc, int64_t M, int64_t N, int64_t K,
                               void* stream) {
    H3B_REQUIRE(fits_int(M) && fits_int(N) && fits_int(K), "h3b_int8_mm_i32: shape out of range");
    gemm::Args a{nullptr, nullptr, nullptr, acc, (int)M, (int)N, (int)K, nullptr};
    return gemm::launch<true>(xq, w, a, static_cast<cudaStream_t>(stream));
}

static int mm_scaled_a2a(const int8_t* xq, const int8_t* w, const float* xs, const float* ws, const void* bias,
                         int64_t M, int64_t N, int64_t K, void* const* dst, int64_t row_start, int64_t seg_cols,
                         int64_t head_dim, int64_t heads_per_rank, int world, const void* norm_w, int64_t norm_segs,
                         float norm_eps, void* stream);

extern "C" int h3b_int8_mm_scaled_a2a(const int8_t* xq, const int8_t* w, const float* xs, const float* ws,
                                      const void* bias, int64_t M, int64_t N, int64_t K, void* const* dst,
                                      int64_t row_start, int64_t seg_cols, int64_t head_dim, int64_t heads_per_rank,
                                      int world, void* stream) {
    return mm_scaled_a2a(xq, w, xs, ws, bias, M, N, K, dst, row_start, seg_cols, head_dim, heads_per_rank, world,
                         nullptr, 0, 0.0f, stream);
}

extern "C" int h3b_int8_mm_scaled_a2a_qknorm(const int8_t* xq, const int8_t* w, const float* xs, const float* ws,
                                             const void* bias, int64_t M, int64_t N, int64_t K, void* const* dst,
                                             int64_t row_start, int64_t seg_cols, int64_t head_dim,
                                             int64_t heads_per_rank, int world, const void* norm_w, int64_t norm_segs,
                                             float norm_eps, void* stream) {
    H3B_REQUIRE(norm_w && norm_segs >= 1 && norm_segs <= N / (seg_cols > 0 ? seg_cols : 1) && head_dim == 128 &&
                    aligned(norm_w, 16),
                "h3b_int8_mm_scaled_a2a_qknorm: norm_w (16-byte aligned, [norm_segs, 128]) and 1 <= norm_segs <= "
                "segments with head_dim 128 required (norm_segs=%lld head_dim=%lld)",
                (long long)norm_segs, (long long)head_dim);
    return mm_scaled_a2a(xq, w, xs, ws, bias, M, N, K, dst, row_start, seg_cols, head_dim, heads_per_rank, world,
                         norm_w, norm_segs, norm_eps, stream);
}

static int mm_scaled_a2a(const int8_t* xq, const int8_t* w, const float* xs, const float* ws, const void* bias,
                         int64_t M, int64_t N, int64_t K, void* const* dst, int64_t row_start, int64_t seg_cols,
                         int64_t head_dim, int64_t heads_per_rank, int world, const void* norm_w, int64_t norm_segs,
                         float norm_eps, void* stream) {
    H3B_REQUIRE(fits_int(M) && fits_int(N) && fits_int(K), "h3b_int8_mm_scaled_a2a: shape out of range");
    H3B_REQUIRE(dst && world >= 1 && world <= gemm::kMaxScatterWorld && row_start >= 0,
                "h3b_int8_mm_scaled_a2a: bad dst / world=%d / row_start", world);
    H3B_REQUIRE(head_dim > 0 && head_dim % 64 == 0 && seg_cols > 0 && seg_cols % head_dim == 0 && N % seg_cols == 0 &&
                    N / seg_cols <= gemm::kMaxScatterSegs && seg_cols / head_dim == heads_per_rank * world,
                "h3b_int8_mm_scaled_a2a: N=%lld seg=%lld head_dim=%lld heads_per_rank=%lld world=%d do not describe "
                "whole heads split evenly over the ranks (head_dim %% 64 == 0, at most %d segments)",
                (long long)N, (long long)seg_cols, (long long)head_dim, (long long)heads_per_rank, world,
                gemm::kMaxScatterSegs);
    gemm::Args a{xs, ws, static_cast<const uint16_t*>(bias), nullptr, (int)M, (int)N, (int)K, nullptr};
    const int segs = (int)(N / seg_cols);
    for (int i = 0; i < segs * world; ++i) {
        H3B_REQUIRE(dst[i] && aligned(dst[i], 16), "h3b_int8_mm_scaled_a2a: dst[%d] NULL or not 16-byte aligned", i);
        a.sc.dst[i] = static_cast<uint16_t*>(dst[i]);
    }
    a.sc.row_start = row_start;
    a.sc.seg = (int)seg_cols;
    a.sc.head_dim = (int)head_dim;
    a.sc.hp = (int)heads_per_rank;
    a.sc.world = world;
    a.sc.norm_w = static_cast<const uint16_t*>(norm_w);
    a.sc.norm_segs = (int)norm_segs;
    a.sc.norm_eps = norm_eps;
    return gemm::launch<false, true>(xq, w, a, static_cast<cudaStream_t>(stream));
}

extern "C" int h3b_int8_linear(const void* x, int64_t M, int64_t K, const int8_t* w, const float* ws,
                               const void* bias, int64_t N, void* out, int8_t* xq_scratch, float* xs_scratch,
                               void* stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    H3B_REQUIRE(K % gemm::BK == 0, "h3b_int8_linear: K=%lld must be a multiple of %d", (long long)K, gemm::BK);
    if (int rc = quant_rowwise(x, K, M, K, xq_scratch, xs_scratch, s)) return rc;
    return h3b_int8_mm_scaled(xq_scratch, w, xs_scratch, ws, bias, out, M, N, K, stream);
}

// ---------------------------------------------------------------------------
// Allocation-free INT8 linear.  Some callers cannot allocate device memory for
// the quantised activations: a C or FFI host that binds this library without
// a device allocator of its own, or a serving loop that must not call
// cudaMalloc (which synchronises the device) in the middle of a step.  For
// them the activation codes and per-row scales live in fixed file-scope
// device arrays.  Every GPU that loads the library holds these arrays
// (8 MiB + 256 KiB) until the process exits; calls beyond their size are
// rejected.  All calls share the arrays, so calls that overlap on the GPU
// (two streams, or two threads) race; the quantiser rewrites every code and
// scale a call reads, so nothing needs clearing between calls.

namespace h3b {
namespace noalloc {

constexpr int64_t kCodesBytes = 8ll << 20;  // M * K int8 activation codes
constexpr int64_t kMaxRows = 65536;         // M fp32 per-row scales

static __device__ __align__(256) int8_t g_codes[kCodesBytes];
static __device__ __align__(256) float g_scales[kMaxRows];

struct Scratch {
    int8_t* codes;
    float* scales;
};

// The host-side names g_codes / g_scales are stand-ins, not device addresses:
// the device addresses are looked up once per device, with that device
// current, on the first call made on it.  The lookup runs under a per-device
// std::call_once, so host threads making their first calls at the same time
// all see both addresses or the lookup's error, never half a result.
constexpr int kMaxDevices = 64;

struct DeviceSlot {
    std::once_flag once;
    Scratch sc{nullptr, nullptr};
    cudaError_t err = cudaSuccess;
};

static int scratch_for_current_device(Scratch* out) {
    static DeviceSlot slots[kMaxDevices];
    int dev = 0;
    H3B_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return set_error(H3B_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
    DeviceSlot& slot = slots[dev];
    std::call_once(slot.once, [&slot] {
        void* c = nullptr;
        void* s = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&c, g_codes);
        if (e == cudaSuccess) e = cudaGetSymbolAddress(&s, g_scales);
        if (e == cudaSuccess) slot.sc = Scratch{static_cast<int8_t*>(c), static_cast<float*>(s)};
        slot.err = e;
    });
    if (slot.err != cudaSuccess) return cuda_error(slot.err, "cudaGetSymbolAddress(noalloc scratch)");
    *out = slot.sc;
    return H3B_OK;
}

}  // namespace noalloc
}  // namespace h3b

extern "C" int h3b_int8_linear_noalloc(const void* x, int64_t M, int64_t K, const int8_t* w, const float* ws,
                                       const void* bias, int64_t N, void* out, void* stream) {
    H3B_REQUIRE(M >= 0 && K > 0 && K % gemm::BK == 0, "h3b_int8_linear_noalloc: K=%lld must be a positive multiple of %d",
                (long long)K, gemm::BK);
    H3B_REQUIRE(M <= noalloc::kMaxRows,
                "h3b_int8_linear_noalloc: M=%lld rows exceed the built-in scale buffer (%lld rows); use h3b_int8_linear",
                (long long)M, (long long)noalloc::kMaxRows);
    H3B_REQUIRE(M * K <= noalloc::kCodesBytes,
                "h3b_int8_linear_noalloc: M*K=%lld exceeds the built-in %lld-byte activation buffer; use h3b_int8_linear",
                (long long)(M * K), (long long)noalloc::kCodesBytes);
    // every host-side check of the allocating path runs before the first CUDA
    // call (the scratch lookup creates the context and loads the module)
    H3B_REQUIRE(x && w && ws && out, "h3b_int8_linear_noalloc: NULL pointer");
    H3B_REQUIRE(aligned(x, 16) && aligned(w, 16) && aligned(out, 16) && aligned(ws, 16) && (!bias || aligned(bias, 16)),
                "h3b_int8_linear_noalloc: x, w, ws, bias and out must be 16-byte aligned");
    H3B_REQUIRE(N > 0 && N % 8 == 0, "h3b_int8_linear_noalloc: N=%lld must be a positive multiple of 8", (long long)N);
    noalloc::Scratch sc;
    if (int rc = noalloc::scratch_for_current_device(&sc)) return rc;
    return h3b_int8_linear(x, M, K, w, ws, bias, N, out, sc.codes, sc.scales, stream);
}
