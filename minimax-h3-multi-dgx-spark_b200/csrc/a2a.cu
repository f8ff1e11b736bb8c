// a10/a11: Ulysses sequence<->head all-to-all layout kernels.
//
// NCCL path: pack [s_local, P*chunk] -> [P, s_local, chunk] before the grouped
// send/recv and unpack [P, s_local, chunk] -> [s_local, P*chunk] after it.
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

// One CTA per source row s; vector e of the row goes to block j = e / cv.
__global__ void __launch_bounds__(256) pack_kernel(const uint4* __restrict__ src, int64_t src_ldv,
                                                   uint4* __restrict__ dst, int64_t s_local, int cv, int world) {
    for (int64_t s = blockIdx.x; s < s_local; s += gridDim.x) {
        const uint4* row = src + s * src_ldv;
        for (int e = threadIdx.x; e < cv * world; e += blockDim.x) {
            const int j = e / cv, v = e - j * cv;
            dst[((int64_t)j * s_local + s) * cv + v] = row[e];
        }
    }
}

__global__ void __launch_bounds__(256) unpack_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst,
                                                     int64_t s_local, int cv, int world) {
    for (int64_t s = blockIdx.x; s < s_local; s += gridDim.x) {
        uint4* row = dst + s * (int64_t)cv * world;
        for (int e = threadIdx.x; e < cv * world; e += blockDim.x) {
            const int j = e / cv, v = e - j * cv;
            row[e] = src[((int64_t)j * s_local + s) * cv + v];
        }
    }
}

struct FwdP2PArgs {
    const uint4* src[kMaxFwdTensors];
    uint4* dst[kMaxFwdTensors][kMaxWorld];
};

// blockIdx.y = tensor.  dst[i][j] row (row_start + s) <- src[i] row s block j.
__global__ void __launch_bounds__(256) fwd_p2p_kernel(FwdP2PArgs a, int64_t src_ldv, int64_t s_local,
                                                      int64_t row_start, int cv, int world) {
    const int i = blockIdx.y;
    const uint4* src = a.src[i];
    for (int64_t s = blockIdx.x; s < s_local; s += gridDim.x) {
        const uint4* row = src + s * src_ldv;
        for (int e = threadIdx.x; e < cv * world; e += blockDim.x) {
            const int j = e / cv, v = e - j * cv;
            a.dst[i][j][(row_start + s) * cv + v] = row[e];
        }
    }
}

struct InvP2PArgs {
    uint4* dst[kMaxWorld];
    int64_t start[kMaxWorld + 1];
};

// Source row q (global sequence index) belongs to rank j with
// start[j] <= q < start[j+1]; it lands in dst[j] row q - start[j], block `rank`.
__global__ void __launch_bounds__(256) inv_p2p_kernel(InvP2PArgs a, const uint4* __restrict__ src, int64_t src_ldv,
                                                      int64_t S, int cv, int world, int rank) {
    for (int64_t q = blockIdx.x; q < S; q += gridDim.x) {
        int j = 0;
        while (j + 1 < world && q >= a.start[j + 1]) ++j;
        const uint4* row = src + q * src_ldv;
        uint4* out = a.dst[j] + ((q - a.start[j]) * world + rank) * (int64_t)cv;
        for (int v = threadIdx.x; v < cv; v += blockDim.x) out[v] = row[v];
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
__global__ void peer_barrier_kernel(BarrierArgs a, int world, int rank, uint32_t epoch, int64_t timeout_ns,
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

static unsigned copy_grid(int64_t rows) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t cap = (int64_t)sms * 16;
    return (unsigned)(rows < cap ? (rows > 0 ? rows : 1) : cap);
}

}  // namespace h3b

using namespace h3b;

extern "C" int h3b_a2a_pack(const void* t, int64_t t_ld, void* send, int64_t s_local, int64_t chunk_bytes,
                            int world, void* stream) {
    H3B_REQUIRE(t && send, "h3b_a2a_pack: NULL pointer");
    H3B_REQUIRE(t_ld >= chunk_bytes * world && t_ld % 16 == 0, "h3b_a2a_pack: t_ld=%lld must be >= a row and a multiple of 16", (long long)t_ld);
    H3B_REQUIRE(world >= 1 && s_local >= 0 && chunk_bytes > 0 && chunk_bytes % 16 == 0 && chunk_bytes * world < (1ll << 31),
                "h3b_a2a_pack: chunk_bytes=%lld must be a positive multiple of 16", (long long)chunk_bytes);
    H3B_REQUIRE(aligned(t, 16) && aligned(send, 16), "h3b_a2a_pack: buffers must be 16-byte aligned");
    if (s_local == 0) return H3B_OK;
    pack_kernel<<<copy_grid(s_local), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint4*>(t), t_ld / 16, static_cast<uint4*>(send), s_local, (int)(chunk_bytes / 16), world);
    H3B_CUDA_TRY(cudaGetLastError());
    return H3B_OK;
}

extern "C" int h3b_a2a_unpack(const void* recv, void* out, int64_t s_local, int64_t chunk_bytes, int world,
                              void* stream) {
    H3B_REQUIRE(recv && out, "h3b_a2a_unpack: NULL pointer");
    H3B_REQUIRE(world >= 1 && s_local >= 0 && chunk_bytes > 0 && chunk_bytes % 16 == 0 && chunk_bytes * world < (1ll << 31),
                "h3b_a2a_unpack: chunk_bytes=%lld must be a positive multiple of 16", (long long)chunk_bytes);
    H3B_REQUIRE(aligned(recv, 16) && aligned(out, 16), "h3b_a2a_unpack: buffers must be 16-byte aligned");
    if (s_local == 0) return H3B_OK;
    unpack_kernel<<<copy_grid(s_local), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint4*>(recv), static_cast<uint4*>(out), s_local, (int)(chunk_bytes / 16), world);
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
                               int64_t row_start, int64_t chunk_bytes, int world, void* stream) {
    H3B_REQUIRE(n >= 1 && n <= kMaxFwdTensors && src && dst, "h3b_a2a_fwd_p2p: bad tensor count %d", n);
    H3B_REQUIRE(world >= 1 && world <= kMaxWorld, "h3b_a2a_fwd_p2p: world=%d out of range", world);
    H3B_REQUIRE(s_local >= 0 && row_start >= 0 && chunk_bytes > 0 && chunk_bytes % 16 == 0 && chunk_bytes * world < (1ll << 31),
                "h3b_a2a_fwd_p2p: chunk_bytes=%lld must be a positive multiple of 16", (long long)chunk_bytes);
    H3B_REQUIRE(src_ld >= chunk_bytes * world && src_ld % 16 == 0, "h3b_a2a_fwd_p2p: src_ld=%lld must be >= a row and a multiple of 16", (long long)src_ld);
    FwdP2PArgs a{};
    for (int i = 0; i < n; ++i) {
        H3B_REQUIRE(src[i] && aligned(src[i], 16), "h3b_a2a_fwd_p2p: src[%d] NULL/misaligned", i);
        a.src[i] = static_cast<const uint4*>(src[i]);
        for (int j = 0; j < world; ++j) {
            H3B_REQUIRE(dst[i * world + j] && aligned(dst[i * world + j], 16), "h3b_a2a_fwd_p2p: dst[%d] NULL/misaligned", i * world + j);
            a.dst[i][j] = static_cast<uint4*>(dst[i * world + j]);
        }
    }
    if (s_local == 0) return H3B_OK;
    dim3 grid(copy_grid(s_local), n);
    fwd_p2p_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(a, src_ld / 16, s_local, row_start,
                                                                         (int)(chunk_bytes / 16), world);
    H3B_CUDA_TRY(cudaGetLastError());
    return H3B_OK;
}

extern "C" int h3b_a2a_inv_p2p(const void* src, int64_t src_ld, void* const* dst, const int64_t* splits,
                               int64_t chunk_bytes, int world, int rank, void* stream) {
    H3B_REQUIRE(src && dst && splits && world >= 1 && world <= kMaxWorld && rank >= 0 && rank < world,
                "h3b_a2a_inv_p2p: bad arguments (world=%d rank=%d)", world, rank);
    H3B_REQUIRE(chunk_bytes > 0 && chunk_bytes % 16 == 0 && src_ld >= chunk_bytes && src_ld % 16 == 0 && aligned(src, 16),
                "h3b_a2a_inv_p2p: chunk_bytes=%lld / src_ld=%lld must be multiples of 16", (long long)chunk_bytes, (long long)src_ld);
    InvP2PArgs a{};
    int64_t S = 0;
    for (int j = 0; j < world; ++j) {
        H3B_REQUIRE(dst[j] && aligned(dst[j], 16) && splits[j] >= 0, "h3b_a2a_inv_p2p: dst[%d]/splits invalid", j);
        a.dst[j] = static_cast<uint4*>(dst[j]);
        a.start[j] = S;
        S += splits[j];
    }
    a.start[world] = S;
    if (S == 0) return H3B_OK;
    inv_p2p_kernel<<<copy_grid(S), 128, 0, static_cast<cudaStream_t>(stream)>>>(
        a, static_cast<const uint4*>(src), src_ld / 16, S, (int)(chunk_bytes / 16), world, rank);
    H3B_CUDA_TRY(cudaGetLastError());
    return H3B_OK;
}
