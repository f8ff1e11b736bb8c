/*
 * h3b.h -- C ABI of libh3b, the B200 (sm_100a) implementation of the H3 video
 * DiT hot path: INT8 linear, fused RMSNorm/adaLN/gate chain, Ulysses
 * sequence<->head all-to-all.
 *
 * Conventions
 *   - Plain device pointers and sizes; no framework types.  bf16 tensors are
 *     passed as `void*` to 16-bit storage.  All tensors are row-major and
 *     contiguous unless a leading dimension is given.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).  Every entry
 *     point only enqueues work; none synchronises unless stated.
 *   - The caller owns every buffer: outputs and scratch are allocated by the
 *     caller (the Python host uses PyTorch's caching allocator), and the
 *     library never frees caller memory.
 *   - Return value: H3B_OK (0) or a negative H3B_ERR_* code;
 *     h3b_last_error() describes the last failure on the calling thread.
 *   - Kernels that wait (mbarrier pipelines, peer flags) give up after a
 *     bounded time and record an H3B_STATUS_* code in a device status word;
 *     read it with h3b_status_get().
 *
 * Reference interfaces cited as path:line inside the reference project
 * (yuichi-suzuki-highdrama/minimax-h3-multi-dgx-spark).
 */
#ifndef H3B_H_
#define H3B_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define H3B_ABI_VERSION 2

#if defined(__GNUC__)
#define H3B_API __attribute__((visibility("default")))
#else
#define H3B_API
#endif

#define H3B_OK 0
#define H3B_ERR_ARG (-1)         /* bad shape, stride, alignment or pointer */
#define H3B_ERR_CUDA (-2)        /* a CUDA runtime/driver call failed */
#define H3B_ERR_UNSUPPORTED (-3) /* not an sm_100 device, or a size the kernels do not cover */

#define H3B_STATUS_OK 0
#define H3B_STATUS_MBAR_TIMEOUT 1 /* a GEMM pipeline wait ran out (kernel aborted its tile loop) */
#define H3B_STATUS_PEER_TIMEOUT 2 /* a peer barrier wait ran out (a rank did not arrive) */
#define H3B_STATUS_BAD_INDEX 3    /* a modulation row index was outside [0, R) (row skipped) */

H3B_API int h3b_abi_version(void);
H3B_API const char *h3b_last_error(void);

/* Device status word of the current device.  h3b_status_get synchronises
 * `stream` first, then reads the word; h3b_status_clear resets it to 0. */
H3B_API int h3b_status_get(int *status_out, void *stream);
H3B_API int h3b_status_clear(void *stream);

/* ---- INT8 linear ------------------------------------------------------- */

/* Per-token absmax activation quantisation (row m of x, leading dimension ldx
 * elements): xs[m] = max_k |x[m,k]| / 127 (IEEE fp32 division);
 * xq[m,k] = clamp(rint_half_even(x[m,k] / xs[m]), -127, 127); an all-zero row
 * gives xs = 0 and xq = 0.  x bf16 [M,K]; xq int8 [M,K]; xs fp32 [M].
 * K % 8 == 0, K <= 32768, x and ldx 16-byte aligned.
 * Replaces comfy-kitchen's _C.quantize_int8_rowwise_convrot64 at the call site
 * comfyui_nodes/h3-linear-fast/h3_linear_fast_patch.py:89-95 (the formula is
 * the plain per-token absmax quantiser; the ConvRot rotation is not applied). */
H3B_API int h3b_quant_rowwise(const void *x, int64_t ldx, int64_t M, int64_t K, int8_t *xq, float *xs, void *stream);

/* The quantiser with the ConvRot rotation: every group of `group` columns
 * (64 or 256; K % group == 0, K <= 32768) of row m is rotated by the normalised
 * Walsh-Hadamard transform y = H x / sqrt(group) (Sylvester order, computed as
 * the fast transform in fp32: stages h = 1, 2, .., group/2, each pair
 * (y_i + y_{i+h}, y_i - y_{i+h}) rounded once, then the exact scale), and y
 * is quantised as by h3b_quant_rowwise: xs[m] = max|y| / 127, xq = rint(y / xs).
 * The weights of such a linear are stored rotated the same way.  Replaces
 * comfy-kitchen 0.2.39's _C.quantize_int8_rowwise_convrot64(x, xq, xs, 256, ...)
 * at comfyui_nodes/h3-linear-fast/h3_linear_fast_patch.py:89-95 (input_act
 * none); that kernel's source is not part of the reference, so its exact
 * arithmetic is not pinned -- this is the rotate-then-quantise scheme it
 * names, with the rounding defined above. */
H3B_API int h3b_quant_rowwise_convrot(const void *x, int64_t ldx, int64_t M, int64_t K, int64_t group, int8_t *xq,
                                      float *xs, void *stream);

/* h3b_quant_rowwise_convrot with the SwiGLU input activation fused in front:
 * x bf16 [M, 2K] (leading dimension ldx elements) holds the gate a = x[:, :K]
 * and the up projection b = x[:, K:]; the row quantised is
 * bf16(silu(a) * b), silu(a) = a / (1 + expf(-a)) in fp32 with one rounding
 * per operation (equal to (F.silu(a.float()) * b.float()).to(bf16) in PyTorch),
 * rotated and quantised exactly as h3b_quant_rowwise_convrot, without the
 * activation reaching memory.  Replaces the reference fast path's fc2 call,
 * _C.quantize_int8_rowwise_convrot64(..., input_act="swiglu"),
 * h3_linear_fast_patch.py:63,89-95 (which half is the gate is not stated in
 * the reference; the first half is the gate here). */
H3B_API int h3b_swiglu_quant_convrot(const void *x, int64_t ldx, int64_t M, int64_t K, int64_t group, int8_t *xq,
                                     float *xs, void *stream);

/* GELU (tanh approximation, PyTorch's fp32 formula) fused into the quantiser:
 * the codes / scales of bf16(gelu(u)) for u bf16 [M,K] (leading dimension ldu)
 * -- the input of the FFN down projection -- without writing the activation.
 * Equals h3b_quant_rowwise(F.gelu(u, approximate="tanh")) bit for bit.  The
 * reference fuses its own activation (SwiGLU) into the quantiser the same way,
 * h3_linear_fast_patch.py:3-5,93-95 (input_act).  The GELU is read from a
 * 65536-entry table (one bf16 output per bf16 input) that the first call on a
 * device fills from that formula and waits for: make that first call before
 * any stream capture.  It and h3b_gelu_tanh share the table. */
H3B_API int h3b_gelu_quant(const void *u, int64_t ldu, int64_t M, int64_t K, int8_t *xq, float *xs, void *stream);

/* y = F.gelu(x, approximate="tanh") on n bf16 elements (n even, x and y
 * 16-byte aligned), bit for bit: the FFN activation between the up and down
 * projections of the block's mlp (the self.mlp call of
 * comfyui_nodes/h3-fuse-graph/h3_fuse_patch.py:133) when it is not fused into
 * the down projection's quantiser.  Reads the table of h3b_gelu_quant (filled
 * by the first call of either on a device). */
H3B_API int h3b_gelu_tanh(const void *x, void *y, int64_t n, void *stream);

/* INT8 GEMM with dequant epilogue on tcgen05 tensor cores:
 * acc[m,n] = sum_k xq[m,k] * w[n,k] (int32), out[m,n] =
 * bf16((float(acc) * xs[m]) * ws[n] [+ float(bias[n])]) with one rounding.
 * xq int8 [M,K], w int8 [N,K] (both K-contiguous), xs fp32 [M], ws fp32 [N],
 * bias bf16 [N] or NULL, out bf16 [M,N].  K % 128 == 0, N % 8 == 0, all
 * pointers 16-byte aligned.
 * Replaces int8_mm_scaled, comfyui_nodes/h3-linear-fast/int8_gemm_triton.py:74-83
 * (kernel :32-66; bias is an addition, NULL reproduces the reference formula). */
H3B_API int h3b_int8_mm_scaled(const int8_t *xq, const int8_t *w, const float *xs, const float *ws, const void *bias,
                       void *out, int64_t M, int64_t N, int64_t K, void *stream);

/* h3b_int8_mm_scaled with the GELU (tanh) of the FFN in the epilogue:
 * out[m,n] = bf16(gelu(y)), y = the bf16 value h3b_int8_mm_scaled would store,
 * gelu in PyTorch's fp32 formula (x^3 as (x*x)*x, inner = kBeta * fma(kKappa,
 * x^3, x), 0.5*x*(1 + tanhf(inner))), each operation rounded once -- equal to
 * F.gelu(h3b_int8_mm_scaled(...), approximate="tanh") bit for bit, without the
 * pre-activation reaching memory.  The up projection + activation of the
 * block's MLP (comfyui_nodes/h3-fuse-graph/h3_fuse_kernels.py:3-7, mlp_out; the
 * reference's checkpoint fuses its SwiGLU into the next quantiser instead,
 * h3_linear_fast_patch.py:63). */
H3B_API int h3b_int8_mm_scaled_gelu(const int8_t *xq, const int8_t *w, const float *xs, const float *ws,
                                    const void *bias, void *out, int64_t M, int64_t N, int64_t K, void *stream);

/* Same GEMM writing the raw int32 accumulators acc [M,N] (the value the
 * reference kernel's tl.dot produces, int8_gemm_triton.py:54-60). */
H3B_API int h3b_int8_mm_i32(const int8_t *xq, const int8_t *w, int32_t *acc, int64_t M, int64_t N, int64_t K,
                    void *stream);

/* h3b_int8_mm_scaled fused with the Ulysses forward all-to-all: instead of
 * out [M,N], the epilogue stores each output column straight into the receive
 * buffer of the rank that owns its head, over NVLink for the other ranks.
 * N = S_g * seg_cols (S_g <= 3 segments: q, k, v of a fused qkv projection);
 * column n belongs to segment t = n / seg_cols and head h = (n % seg_cols) /
 * head_dim, owned by rank j = h / heads_per_rank; it is stored to
 * dst[t * world + j] (bf16, rows of heads_per_rank * head_dim elements; at
 * least row_start + M rows) at row row_start + m, column
 * (h - j * heads_per_rank) * head_dim + n % head_dim -- exactly what
 * h3b_a2a_fwd_p2p delivers after an unfused GEMM, value for value.
 * head_dim % 64 == 0, seg_cols == world * heads_per_rank * head_dim,
 * world <= 8.  Bracket with h3b_peer_barrier like the exchange it replaces.
 * Replaces the qkv projection + a2a_gather_seq_scatter_heads (x3) of
 * sp_attention, comfyui_nodes/minimax-h3-sp/minimax_sp/sp_forward.py:284,308-311. */
H3B_API int h3b_int8_mm_scaled_a2a(const int8_t *xq, const int8_t *w, const float *xs, const float *ws,
                                   const void *bias, int64_t M, int64_t N, int64_t K, void *const *dst,
                                   int64_t row_start, int64_t seg_cols, int64_t head_dim, int64_t heads_per_rank,
                                   int world, void *stream);

/* h3b_int8_mm_scaled_a2a with the attention's per-head q / k RMSNorm in the
 * epilogue: every 128-column head of the first norm_segs segments (q, then k)
 * of each row becomes rbf16(w_t * (rstd * y)), rstd = rsqrt(sum(y^2)/128 + eps),
 * y the bf16 projection output and w_t = norm_w + t * 128 (bf16 [norm_segs, 128]),
 * with the reduction order of h3b_rms_norm / F.rms_norm, before it is stored
 * into the owning rank's receive buffer.  head_dim == 128.  Replaces the qkv
 * projection, attn.q_norm / attn.k_norm and the forward exchange of
 * sp_attention, sp_forward.py:280-284,296-298,308-311 (the no-RoPE branch). */
H3B_API int h3b_int8_mm_scaled_a2a_qknorm(const int8_t *xq, const int8_t *w, const float *xs, const float *ws,
                                          const void *bias, int64_t M, int64_t N, int64_t K, void *const *dst,
                                          int64_t row_start, int64_t seg_cols, int64_t head_dim,
                                          int64_t heads_per_rank, int world, const void *norm_w, int64_t norm_segs,
                                          float norm_eps, void *stream);

/* Patched Linear forward: quantise x (h3b_quant_rowwise) into the caller's
 * scratch xq [M,K] / xs [M], then h3b_int8_mm_scaled into out [M,N].
 * Replaces the patched comfy_kitchen.backends.cuda.int8_linear,
 * comfyui_nodes/h3-linear-fast/h3_linear_fast_patch.py:60-110. */
H3B_API int h3b_int8_linear(const void *x, int64_t M, int64_t K, const int8_t *w, const float *ws, const void *bias,
                    int64_t N, void *out, int8_t *xq_scratch, float *xs_scratch, void *stream);

/* h3b_int8_linear without caller-provided scratch, for callers that cannot
 * allocate device memory (a C/FFI host with no device allocator of its own,
 * or a serving loop that must not call cudaMalloc mid-step).  The int8 codes
 * and row scales go to fixed device arrays inside the library: M * K <= 8 MiB
 * and M <= 65536, larger calls are rejected with H3B_ERR_ARG.  Each GPU that
 * loads the library holds those 8.25 MiB until exit.  The first call on a
 * device looks up the arrays' device addresses (make it before any stream
 * capture).  Calls share the arrays: calls that overlap on the GPU race.
 * No counterpart in the reference, which always allocates its activation
 * codes and scales; this entry point allocates nothing itself. */
H3B_API int h3b_int8_linear_noalloc(const void *x, int64_t M, int64_t K, const int8_t *w, const float *ws,
                                    const void *bias, int64_t N, void *out, void *stream);

/* ---- fused RMSNorm / adaLN modulation / gate / residual ----------------- */
/* x, o, h bf16 [S,D]; w bf16 [D]; ridx int32 [S] selects a row of the bf16
 * modulation tables s1 / sh / g [R,D] (0 <= ridx < R is checked on the
 * device: a row with an out-of-range index is skipped and recorded as
 * H3B_STATUS_BAD_INDEX).  D % 4 == 0, D <= 16384,
 * rows 8-byte aligned.  Sums of squares, the rsqrt and the bf16 rounding
 * points follow the reference kernels bit for bit (rsqrtf as on the GPU). */

/* h = bf16(rbf16(rbf16(w * (rstd * x)) * s1[r]) + sh[r]),
 * rstd = rsqrt(sum(x^2) / D + eps).
 * Replaces norm_mod, comfyui_nodes/h3-fuse-graph/h3_fuse_kernels.py:174-178 (kernel :88-114). */
H3B_API int h3b_norm_mod(const void *x, const void *w, float eps, const int32_t *ridx, const void *s1, const void *sh,
                 void *h, int64_t S, int64_t D, int64_t R, void *stream);

/* Plain RMSNorm with a weight, no modulation: h = rbf16(w * (rstd * x)),
 * rstd = rsqrt(sum(x^2) / D + eps), the same reduction order and rounding as
 * h3b_norm_mod's first step (PyTorch's F.rms_norm(x, (D,), w, eps)).  x, h bf16
 * [S, D], w bf16 [D], D % 8 == 0, 16-byte aligned.  Covers the per-head q/k norm
 * of sp_attention when it has no RoPE (x = [S*H, head_dim]),
 * comfyui_nodes/minimax-h3-sp/minimax_sp/sp_forward.py:296-298. */
H3B_API int h3b_rms_norm(const void *x, const void *w, float eps, void *h, int64_t S, int64_t D, void *stream);

/* x <- bf16(x + o * g[r]) in place, then h = norm_mod(x).
 * Replaces gate_norm_mod_, h3_fuse_kernels.py:181-185 (kernel :117-155). */
H3B_API int h3b_gate_norm_mod_(void *x, const void *o, const void *g, const void *w, float eps, const int32_t *ridx,
                       const void *s1, const void *sh, void *h, int64_t S, int64_t D, int64_t R, void *stream);

/* norm_mod fused with the activation quantiser of the linear it feeds:
 * instead of h, writes xq int8 [S,D] and xs fp32 [S] equal to
 * h3b_quant_rowwise(h3b_norm_mod(...)) bit for bit (h never reaches HBM).
 * D % 8 == 0, 16-byte aligned tensors.  Replaces the pair norm_mod
 * (h3_fuse_kernels.py:174-178) -> quantiser call (h3_linear_fast_patch.py:89-95)
 * at h3_fuse_patch.py:125 + sp_forward.py:280. */
H3B_API int h3b_norm_mod_quant(const void *x, const void *w, float eps, const int32_t *ridx, const void *s1,
                               const void *sh, int8_t *xq, float *xs, int64_t S, int64_t D, int64_t R, void *stream);

/* gate_norm_mod_ fused with the quantiser: x <- bf16(x + o*g[r]) in place,
 * then the int8 codes / scales of norm_mod(x) (h3_fuse_kernels.py:181-185 ->
 * h3_linear_fast_patch.py:89-95, the MLP input at h3_fuse_patch.py:133-135). */
H3B_API int h3b_gate_norm_mod_quant_(void *x, const void *o, const void *g, const void *w, float eps,
                                     const int32_t *ridx, const void *s1, const void *sh, int8_t *xq, float *xs,
                                     int64_t S, int64_t D, int64_t R, void *stream);

/* x <- bf16(x + o * g[r]) in place.
 * Replaces gate_, h3_fuse_kernels.py:188-192 (kernel :158-167). */
H3B_API int h3b_gate_(void *x, const void *o, const void *g, const int32_t *ridx, int64_t S, int64_t D, int64_t R,
              void *stream);

/* ---- Ulysses all-to-all -------------------------------------------------- */

/* Forward pack: rows of t (row stride t_ld bytes) hold one block of
 * block_bytes per destination rank; the first chunk_bytes of block j of row s
 * go to send[j, s, :] (send is [P, s_local, chunk]).  block = chunk is the
 * whole exchange (t [s_local, P * chunk], chunk = (H/P)*Dh elements); a head
 * group of each rank's heads is a narrower chunk with t offset to the group's
 * first column.  The NCCL exchange that follows receives [S, chunk] already in
 * sequence order.
 * Replaces t.reshape(s_local, p, chunk).transpose(0, 1).contiguous() of
 * comfyui_nodes/minimax-h3-sp/minimax_sp/sp_forward.py:185 and the per-group
 * prep() of sp_attention_overlap, sp_forward.py:222-224. */
H3B_API int h3b_a2a_pack(const void *t, int64_t t_ld, void *send, int64_t s_local, int64_t chunk_bytes,
                         int64_t block_bytes, int world, void *stream);

/* Inverse unpack: recv [P, s_local, chunk] -> row s of out (row stride out_ld
 * bytes), bytes [j*block, j*block + chunk) <- recv[j, s, :].  block = chunk,
 * out_ld = P*chunk is out [s_local, P * chunk]; a head group writes a narrower
 * chunk at its column offset (out offset by the caller).
 * Replaces out.view(p, s_local, chunk).transpose(0, 1).reshape(...) of
 * sp_forward.py:198 and final[:, :, i] = ... of sp_forward.py:257-258. */
H3B_API int h3b_a2a_unpack(const void *recv, void *out, int64_t out_ld, int64_t s_local, int64_t chunk_bytes,
                           int64_t block_bytes, int world, void *stream);

/* Inverse exchange fused with the activation quantiser of the attention
 * output projection: local row m (of M) is the concatenation over ranks
 * j = 0 .. P-1 of row row_start + m of src[j] (rank j's attention output
 * [S, chunk], bf16, rows src_ld bytes apart; a peer's memory for j != this
 * rank), i.e. the row the inverse exchange would deliver; it is quantised
 * exactly as h3b_quant_rowwise (K = P * chunk_bytes / 2 <= 32768) into
 * xq [M, K] / xs [M].  Bracket with h3b_peer_barrier (every src complete).
 * Replaces a2a_scatter_seq_gather_heads, sp_forward.py:191-198, followed by the
 * out projection's quantisation, h3_linear_fast_patch.py:89-95. */
H3B_API int h3b_a2a_inv_quant(const void *const *src, int64_t src_ld, int64_t row_start, int64_t M,
                              int64_t chunk_bytes, int world, int8_t *xq, float *xs, void *stream);

/* CUDA IPC plumbing for the peer-memory all-to-all.  h3b_ipc_handle returns
 * the 64-byte cudaIpcMemHandle of the allocation holding dev_ptr and
 * dev_ptr's offset inside it; h3b_ipc_open maps a peer's allocation and
 * returns base + offset (and the base, for h3b_ipc_close). */
H3B_API int h3b_ipc_handle(const void *dev_ptr, void *handle_out, int64_t *offset_out);
H3B_API int h3b_ipc_open(const void *handle, int64_t offset, void **dev_ptr_out, void **base_out);
H3B_API int h3b_ipc_close(void *base);

/* Cross-rank barrier over peer memory: rank `rank` stores `epoch` into slot
 * [rank] of every peer's flag array (peer_flags[j], uint32 [P]) with
 * system-scope release, then waits until every slot of its own array
 * (peer_flags[rank]) is >= epoch.  Gives up after timeout_ns and records
 * H3B_STATUS_PEER_TIMEOUT.  Work before the barrier on `stream` (including
 * peer-memory stores) is visible to every rank's work after it.
 * Takes the place of the synchronisation inside the NCCL all_to_all_single
 * calls of comfyui_nodes/minimax-h3-sp/minimax_sp/sp_forward.py:164-166,174-176. */
H3B_API int h3b_peer_barrier(uint32_t *const *peer_flags, int world, int rank, uint32_t epoch, int64_t timeout_ns,
                     void *stream);

/* Forward exchange fused with the pack, over peer memory: for each of n
 * tensors src[i] (rows of s_local, row stride src_ld bytes shared by all n)
 * holding one block of block_bytes per destination rank j, the width_bytes at
 * offset_bytes inside block j go straight into rank j's receive buffer
 * dst[i * P + j] (rows of width_bytes) at rows row_start .. row_start + s_local.
 * block = width, offset = 0 is the whole exchange; a head group of the heads
 * rank j owns is a narrower width at an offset.  Bracket with h3b_peer_barrier.
 * Replaces a2a_gather_seq_scatter_heads / _seq_gather, sp_forward.py:158-166,179-188,
 * and the per-group exchanges of sp_attention_overlap, sp_forward.py:211-261. */
H3B_API int h3b_a2a_fwd_p2p(int n, const void *const *src, int64_t src_ld, void *const *dst, int64_t s_local,
                            int64_t row_start, int64_t width_bytes, int64_t block_bytes, int64_t offset_bytes,
                            int world, void *stream);

/* Inverse exchange fused with the unpack: src rows of width_bytes (leading
 * dimension src_ld bytes, S = sum(splits) rows) split by `splits` (P entries)
 * go to rank j's output dst[j] (rows dst_ld bytes apart) at byte column
 * offset_bytes.  For the whole exchange: width = (H/P)*Dh*elt, dst_ld = P*width,
 * offset = rank*width; a head group shifts the offset inside rank's block.
 * Replaces a2a_scatter_seq_gather_heads / _seq_scatter, sp_forward.py:169-176,191-198. */
H3B_API int h3b_a2a_inv_p2p(const void *src, int64_t src_ld, void *const *dst, const int64_t *splits,
                            int64_t width_bytes, int64_t dst_ld, int64_t offset_bytes, int world, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* H3B_H_ */
