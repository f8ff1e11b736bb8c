// a10/a11: Ulysses sequence<->head all-to-all layout kernels.
//
// NCCL path: pack [s_local, P*chunk] -> [P, s_local, chunk] before the grouped
// send/recv and unpack [P, s_local, chunk] -> [s_local, P*chunk] after it
// (or one head group of each rank's chunk: a narrower chunk at a column offset,
// for the exchange/attention overlap).
// Peer-memory path: the pack (forward) and the unpack (inverse) are fused with
// the exchange -- each CTA reads local rows and stores them straight into the
// destination rank's buffer over NVLink, so no staging buffer exists and each
// byte crosses HBM once on each side.  The exchange is bracketed by
// h3b_peer_barrier (flags in peer memory, bounded waits).
// All kernels move 16-byte vectors; chunk sizes must be multiples of 16 bytes.
#include "common.cuh"

namespace h3b {

constexpr int kMaxWorld = 8;
constexpr int kMaxFwdTensors = 4;

// Pack: send[j, s, v] = row s of src, vector j*blk + v (v < w).  blk = w is
// the plain [s_local, P*chunk] -> [P, s_local, chunk] pack; blk > w packs one
// head group (the caller offsets src to the group's first column).
// Flat grid-stride loop over (row, rank, vector); total = s_local*world*w < 2^31.
__global__ void __launch_bounds__(256) pack_kernel(const uint4* __restrict__ src, int64_t src_ldv,
                                                   uint4* __restrict__ dst, uint32_t s_local, uint32_t w,
                                                   uint32_t blk, uint32_t world) {
    const uint32_t rw = w * world, total = s_local * rw;
    for (uint32_t e = blockIdx.x * blockDim.x + threadIdx.x; e < total; e += gridDim.x * blockDim.x) {
        const uint32_t s = e / rw, r = e - s * rw, j = r / w, v = r - j * w;
        dst[((int64_t)j * s_local + s) * w + v] = src[s * src_ldv + j * blk + v];
    }
}

// Unpack: row s of dst (dst_ldv vectors apart), vector j*blk + v <- recv[j, s, v].
__global__ void __launch_bounds__(256) unpack_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst,
                                                     int64_t dst_ldv, uint32_t s_local, uint32_t w, uint32_t blk,
                                                     uint32_t world) {
    const uint32_t rw = w * world, total = s_local * rw;
    for (uint32_t e = blockIdx.x * blockDim.x + threadIdx.x; e < total; e += gridDim.x * blockDim.x) {
        const uint32_t s = e / rw, r = e - s * rw, j = r / w, v = r - j * w;
        dst[s * dst_ldv + j * blk + v] = src[((int64_t)j * s_local + s) * w + v];
    }
}

struct FwdP2PArgs {
    const uint4* src[kMaxFwdTensors];
    uint4* dst[kMaxFwdTensors][kMaxWorld];
};

// blockIdx.y = tensor.  Row s of src[i] holds one block per destination rank j
// starting at vector j*blk + off; w vectors of it go to dst[i][j] row
// (row_start + s) (receive rows are w vectors wide).  With blk = w, off = 0
// this is the plain pack; a head group of the block is blk > w, off > 0.
// Flat grid-stride loop over (row, rank, vector) so that narrow head groups
// (w = 16 vectors for one 128-wide bf16 head) still keep every thread busy;
// total = s_local * world * w < 2^31 (host-checked).
__global__ void __launch_bounds__(256) fwd_p2p_kernel(FwdP2PArgs a, int64_t src_ldv, uint32_t total, int64_t row_start,
                                                      uint32_t w, uint32_t blk, uint32_t off, uint32_t world) {
    const int i = blockIdx.y;
    const uint4* __restrict__ src = a.src[i];
    const uint32_t rw = w * world;
    for (uint32_t e = blockIdx.x * blockDim.x + threadIdx.x; e < total; e += gridDim.x * blockDim.x) {
        const uint32_t s = e / rw, r = e - s * rw, j = r / w, v = r - j * w;
        a.dst[i][j][(row_start + s) * w + v] = src[s * src_ldv + off + j * blk + v];
    }
}

struct InvP2PArgs {
    uint4* dst[kMaxWorld];
    int64_t start[kMaxWorld + 1];
};

// Source row q (global sequence index, w vectors) belongs to rank j with
// start[j] <= q < start[j+1]; it lands in dst[j] row q - start[j] (rows
// dst_ldv vectors apart) at vector column off.  total = S * w < 2^31.
__global__ void __launch_bounds__(256) inv_p2p_kernel(InvP2PArgs a, const uint4* __restrict__ src, int64_t src_ldv,
                                                      uint32_t total, uint32_t w, int64_t dst_ldv, uint32_t off,
                                                      int world) {
    for (uint32_t e = blockIdx.x * blockDim.x + threadIdx.x; e < total; e += gridDim.x * blockDim.x) {
        const uint32_t q = e / w, v = e - q * w;
        int j = 0;
        while (j + 1 < world && (int64_t)q >= a.start[j + 1]) ++j;
        a.dst[j][((int64_t)q - a.start[j]) * dst_ldv + off + v] = src[q * src_ldv + v];
    }
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

struct BarrierArgs {
    uint32_t* flags[kMaxWorld];  // flags[j] = rank j's flag array (uint32 [world])
};

// Thread j signals rank j (slot [rank] of its array) and then waits for rank
// j's signal in slot [j] of this rank's array.  Bounded by timeout_ns.
__global__ void peer_barrier_kernel(const __grid_constant__ BarrierArgs a, int world, int rank, uint32_t epoch, int64_t timeout_ns,
                                    int* status) {
    const int j = threadIdx.x;
    if (j >= world) return;
    __threadfence_system();
    st_release_sys(a.flags[j] + rank, epoch);
    const uint32_t* mine = a.flags[rank] + j;
    const uint64_t t0 = globaltimer_ns();
    uint32_t spins = 0;
    while ((int32_t)(ld_acquire_sys(mine) - epoch) < 0) {
        if ((++spins & 63u) == 0 && (int64_t)(globaltimer_ns() - t0) > timeout_ns) {
            report(status, H3B_STATUS_PEER_TIMEOUT);
            break;
        }
        __nanosleep(64);
    }
    __threadfence_system();
}

static int sm_count() {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}

// Flat copies: 256 threads per CTA, one 16-byte vector per thread per pass,
// at most 8 CTAs per SM.
static unsigned flat_grid(int64_t vectors) {
    const int64_t need = (vectors + 255) / 256, cap = (int64_t)sm_count() * 8;
    return (unsigned)(need < cap ? (need > 0 ? need : 1) : cap);
}

}  // namespace h3b

using namespace h3b;

extern "C" int h3b_a2a_pack(const void* t, int64_t t_ld, void* send, int64_t s_local, int64_t chunk_bytes,
                            int64_t block_bytes, int world, void* stream) {
    H3B_REQUIRE(t && send, "h3b_a2a_pack: NULL pointer");
    H3B_REQUIRE(world >= 1 && world <= kMaxWorld && s_local >= 0 && chunk_bytes > 0 && chunk_bytes % 16 == 0 &&
                    block_bytes % 16 == 0 && block_bytes >= chunk_bytes,
                "h3b_a2a_pack: chunk %lld / block %lld bytes must be multiples of 16 with chunk <= block (world=%d)",
                (long long)chunk_bytes, (long long)block_bytes, world);
    H3B_REQUIRE(t_ld >= block_bytes * (world - 1) + chunk_bytes && t_ld % 16 == 0,
                "h3b_a2a_pack: t_ld=%lld must cover a row and be a multiple of 16", (long long)t_ld);
    H3B_REQUIRE(aligned(t, 16) && aligned(send, 16), "h3b_a2a_pack: buffers must be 16-byte aligned");
    const int64_t total = s_local * world * (chunk_bytes / 16);
    H3B_REQUIRE(total < (1ll << 31), "h3b_a2a_pack: %lld vectors exceed 2^31", (long long)total);
    if (total == 0) return H3B_OK;
    pack_kernel<<<flat_grid(total), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint4*>(t), t_ld / 16, static_cast<uint4*>(send), (uint32_t)s_local,
        (uint32_t)(chunk_bytes / 16), (uint32_t)(block_bytes / 16), (uint32_t)world);
    H3B_CUDA_TRY(cudaGetLastError());
    return H3B_OK;
}

extern "C" int h3b_a2a_unpack(const void* recv, void* out, int64_t out_ld, int64_t s_local, int64_t chunk_bytes,
                              int64_t block_bytes, int world, void* stream) {
    H3B_REQUIRE(recv && out, "h3b_a2a_unpack: NULL pointer");
    H3B_REQUIRE(world >= 1 && world <= kMaxWorld && s_local >= 0 && chunk_bytes > 0 && chunk_bytes % 16 == 0 &&
                    block_bytes % 16 == 0 && block_bytes >= chunk_bytes,
                "h3b_a2a_unpack: chunk %lld / block %lld bytes must be multiples of 16 with chunk <= block (world=%d)",
                (long long)chunk_bytes, (long long)block_bytes, world);
    H3B_REQUIRE(out_ld >= block_bytes * (world - 1) + chunk_bytes && out_ld % 16 == 0,
                "h3b_a2a_unpack: out_ld=%lld must cover a row and be a multiple of 16", (long long)out_ld);
    H3B_REQUIRE(aligned(recv, 16) && aligned(out, 16), "h3b_a2a_unpack: buffers must be 16-byte aligned");
    const int64_t total = s_local * world * (chunk_bytes / 16);
    H3B_REQUIRE(total < (1ll << 31), "h3b_a2a_unpack: %lld vectors exceed 2^31", (long long)total);
    if (total == 0) return H3B_OK;
    unpack_kernel<<<flat_grid(total), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint4*>(recv), static_cast<uint4*>(out), out_ld / 16, (uint32_t)s_local,
        (uint32_t)(chunk_bytes / 16), (uint32_t)(block_bytes / 16), (uint32_t)world);
    H3B_CUDA_TRY(cudaGetLastError());
    return H3B_OK;
}

extern "C" int h3b_peer_barrier(uint32_t* const* peer_flags, int world, int rank, uint32_t epoch,
                                int64_t timeout_ns, void* stream) {
    H3B_REQUIRE(peer_flags && world >= 1 && world <= kMaxWorld && rank >= 0 && rank < world,
                "h3b_peer_barrier: bad world=%d rank=%d", world, rank);
    H3B_REQUIRE(timeout_ns > 0, "h3b_peer_barrier: timeout_ns must be positive");
    BarrierArgs a{};
    for (int j = 0; j < world; ++j) {
        H3B_REQUIRE(peer_flags[j] && aligned(peer_flags[j], 4), "h3b_peer_barrier: flag array %d NULL/misaligned", j);
        a.flags[j] = peer_flags[j];
    }
    DeviceStatus ds;
    if (int rc = device_status(&ds)) return rc;
    peer_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(a, world, rank, epoch, timeout_ns, ds.word);
    H3B_CUDA_TRY(cudaGetLastError());
    return H3B_OK;
}

extern "C" int h3b_a2a_fwd_p2p(int n, const void* const* src, int64_t src_ld, void* const* dst, int64_t s_local,
                               int64_t row_start, int64_t width_bytes, int64_t block_bytes, int64_t offset_bytes,
                               int world, void* stream) {
    H3B_REQUIRE(n >= 1 && n <= kMaxFwdTensors && src && dst, "h3b_a2a_fwd_p2p: bad tensor count %d", n);
    H3B_REQUIRE(world >= 1 && world <= kMaxWorld, "h3b_a2a_fwd_p2p: world=%d out of range", world);
    H3B_REQUIRE(s_local >= 0 && row_start >= 0 && width_bytes > 0 && width_bytes % 16 == 0 && block_bytes % 16 == 0 &&
                    offset_bytes % 16 == 0 && offset_bytes >= 0 && offset_bytes + width_bytes <= block_bytes &&
                    block_bytes * world < (1ll << 31),
                "h3b_a2a_fwd_p2p: width %lld / block %lld / offset %lld bytes must be multiples of 16 with "
                "offset + width <= block", (long long)width_bytes, (long long)block_bytes, (long long)offset_bytes);
    H3B_REQUIRE(src_ld >= block_bytes * world && src_ld % 16 == 0,
                "h3b_a2a_fwd_p2p: src_ld=%lld must be >= a row and a multiple of 16", (long long)src_ld);
    FwdP2PArgs a{};
    for (int i = 0; i < n; ++i) {
        H3B_REQUIRE(src[i] && aligned(src[i], 16), "h3b_a2a_fwd_p2p: src[%d] NULL/misaligned", i);
        a.src[i] = static_cast<const uint4*>(src[i]);
        for (int j = 0; j < world; ++j) {
            H3B_REQUIRE(dst[i * world + j] && aligned(dst[i * world + j], 16), "h3b_a2a_fwd_p2p: dst[%d] NULL/misaligned", i * world + j);
            a.dst[i][j] = static_cast<uint4*>(dst[i * world + j]);
        }
    }
    const int64_t total = s_local * world * (width_bytes / 16);
    H3B_REQUIRE(total < (1ll << 31), "h3b_a2a_fwd_p2p: %lld vectors per tensor exceed 2^31", (long long)total);
    if (total == 0) return H3B_OK;
    dim3 grid(flat_grid(total), n);
    fwd_p2p_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        a, src_ld / 16, (uint32_t)total, row_start, (uint32_t)(width_bytes / 16), (uint32_t)(block_bytes / 16),
        (uint32_t)(offset_bytes / 16), (uint32_t)world);
    H3B_CUDA_TRY(cudaGetLastError());
    return H3B_OK;
}

extern "C" int h3b_a2a_inv_p2p(const void* src, int64_t src_ld, void* const* dst, const int64_t* splits,
                               int64_t width_bytes, int64_t dst_ld, int64_t offset_bytes, int world, void* stream) {
    H3B_REQUIRE(src && dst && splits && world >= 1 && world <= kMaxWorld, "h3b_a2a_inv_p2p: bad arguments (world=%d)", world);
    H3B_REQUIRE(width_bytes > 0 && width_bytes % 16 == 0 && src_ld >= width_bytes && src_ld % 16 == 0 && aligned(src, 16),
                "h3b_a2a_inv_p2p: width %lld / src_ld %lld bytes must be multiples of 16", (long long)width_bytes,
                (long long)src_ld);
    H3B_REQUIRE(dst_ld % 16 == 0 && offset_bytes % 16 == 0 && offset_bytes >= 0 && offset_bytes + width_bytes <= dst_ld,
                "h3b_a2a_inv_p2p: dst_ld %lld / offset %lld bytes must be multiples of 16 with offset + width <= dst_ld",
                (long long)dst_ld, (long long)offset_bytes);
    InvP2PArgs a{};
    int64_t S = 0;
    for (int j = 0; j < world; ++j) {
        H3B_REQUIRE(dst[j] && aligned(dst[j], 16) && splits[j] >= 0, "h3b_a2a_inv_p2p: dst[%d]/splits invalid", j);
        a.dst[j] = static_cast<uint4*>(dst[j]);
        a.start[j] = S;
        S += splits[j];
    }
    a.start[world] = S;
    const int64_t total = S * (width_bytes / 16);
    H3B_REQUIRE(total < (1ll << 31), "h3b_a2a_inv_p2p: %lld vectors exceed 2^31", (long long)total);
    if (total == 0) return H3B_OK;
    inv_p2p_kernel<<<flat_grid(total), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        a, static_cast<const uint4*>(src), src_ld / 16, (uint32_t)total, (uint32_t)(width_bytes / 16), dst_ld / 16,
        (uint32_t)(offset_bytes / 16), world);
    H3B_CUDA_TRY(cudaGetLastError());
    return H3B_OK;
}
