/*
 * genie_tk_b200 -- C ABI of the B200 (sm_100a) triangle hot path.
 *
 * This is the drop-in replacement for the reference's native boundary, the pybind11
 * module `genie_tk._C` declared in kernels/bindings.cpp:13-65 and bound at
 * kernels/bindings.cpp:69-101 of northws/Genie-TK. Plain C types only: device
 * pointers, sizes and an opaque CUDA stream (`cudaStream_t` passed as `void*`).
 *
 * Conventions
 *  - Every entry point returns GTK_OK (0) or a negative GTK_ERR_* code; the message
 *    of the last failure on the calling thread is gtk_last_error_string().
 *  - The caller owns all memory. Outputs, packed weights and workspaces are allocated
 *    by the caller (sizes from the *_bytes queries); the library never allocates
 *    device memory and never synchronises the device. Work is enqueued on `stream`.
 *  - Pair tensors use the reference layout [B, N, N, C], row-major, fp32; masks are
 *    fp32 [B, N, N] (NULL = all ones); parameters are the fp32 nn.Linear / LayerNorm
 *    tensors of the reference modules ([out, in] weights).
 *  - `status` (optional, may be NULL) is a device uint32 word. A kernel whose bounded
 *    wait ran out, or that had to clamp an fp16 intermediate, ORs a GTK_STATUS_* bit into
 *    it and finishes cleanly instead of hanging or failing silently. Read it after
 *    synchronising the stream.
 *  - Shapes: the multiplicative update with c_z = 128, c_hidden <= 128, attention with
 *    c_in = 128 and 4 heads of head_dim <= 32, and the transition with c_p = 128, n <= 4
 *    run on the tuned tcgen05 kernels (narrower hidden widths and head dims are
 *    zero-padded in the packed weights, which changes no result). Every other shape the
 *    reference's modules accept -- channel counts 1..512, attention heads 1..32 with
 *    head_dim = c_hidden / heads <= 64, a transition hidden width <= 2048 -- runs on the
 *    general-shape kernels behind the same forward entry points (the stage entry points
 *    below are the tuned shape only). Beyond those limits GTK_ERR_UNSUPPORTED. Any B >= 1
 *    and N >= 1.
 *  - Thread safety: entry points may be called concurrently on different streams.
 */
#ifndef GENIE_TK_B200_H_
#define GENIE_TK_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define GTK_API __attribute__((visibility("default")))
#else
#define GTK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define GTK_OK 0
#define GTK_ERR_INVALID_ARG (-1)
#define GTK_ERR_UNSUPPORTED (-2)
#define GTK_ERR_ALIGNMENT (-3)
#define GTK_ERR_WORKSPACE (-4)
#define GTK_ERR_CUDA (-5)
#define GTK_ERR_TMAP (-6)
#define GTK_ERR_DEVICE (-7)

#define GTK_STATUS_TIMEOUT_PRODUCER 0x1u
#define GTK_STATUS_TIMEOUT_MMA 0x2u
#define GTK_STATUS_TIMEOUT_CONSUMER 0x4u
#define GTK_STATUS_TIMEOUT_DRAIN 0x8u
#define GTK_STATUS_TIMEOUT_PEER 0x20u /* a cross-GPU barrier ran out: a peer never arrived */
/* An fp16 intermediate (a/b/x planes of the multiplicative update; the LayerNorm output,
 * q, k, v and gated output of attention; the transition's hidden rows) was beyond
 * +-65504 and was clamped, so the result is not the reference's. The tensor-core operands
 * are fp16 (11 significant bits, 3 more than bf16) and in range for LayerNorm-normalised
 * inputs and weights of the usual 1/fan_in scale; inputs or weights large enough to leave
 * that range set this bit instead of returning a silently wrong answer. */
#define GTK_STATUS_FP16_SATURATED 0x40u

/* Library version (major*10000 + minor*100 + patch). */
GTK_API int gtk_version(void);

/* Message of the last failed call on this thread ("" if none). */
GTK_API const char* gtk_last_error_string(void);

/* ---------------------------------------------------------------------------------
 * Triangle multiplicative update (Algorithms 11/12).
 * Replaces `_C.triangle_mul_outgoing` / `_C.triangle_mul_incoming`
 * (kernels/bindings.cpp:16-26, bound at :73-79) together with the PyTorch glue
 * around them in `TriangleMultiplicativeUpdate._forward_cuda`
 * (src/genie_tk/triangle_mul.py:134-169): LN_in, gated masked projections,
 * the per-channel contraction, LN_out, linear_z and the output gate.
 * ------------------------------------------------------------------------------- */

/* fp32 device pointers to the parameters of a reference TriangleMultiplicativeUpdate
 * (src/genie_tk/triangle_mul.py:64-73); weights [out, in]. */
typedef struct gtk_trimul_params {
  const float* ln_in_w;
  const float* ln_in_b;
  const float* a_p_w;
  const float* a_p_b;
  const float* a_g_w;
  const float* a_g_b;
  const float* b_p_w;
  const float* b_p_b;
  const float* b_g_w;
  const float* b_g_b;
  const float* g_w;
  const float* g_b;
  const float* z_w;
  const float* z_b;
  const float* ln_out_w;
  const float* ln_out_b;
} gtk_trimul_params;

/* Bytes of the packed (bf16 / folded) weight buffer. */
GTK_API size_t gtk_trimul_packed_bytes(int c_z, int c_hidden);

/* Convert module parameters into the packed buffer the kernels read. Re-run after
 * the parameters change. `packed` must be 256-B aligned. */
GTK_API int gtk_trimul_pack(const gtk_trimul_params* params, int c_z, int c_hidden, void* packed, size_t packed_bytes,
                    void* stream);

/* Bytes of scratch space gtk_trimul_forward needs for (B, N). */
GTK_API size_t gtk_trimul_workspace_bytes(int64_t B, int64_t N, int c_z, int c_hidden);

/* out = update(z)                 (add_residual = 0; the reference module's return value)
 * out = z + update(z)             (add_residual = 1; out may equal z for in-place use)
 * outgoing = 1: x_ij = sum_k a_ik b_jk; outgoing = 0: x_ij = sum_k a_ki b_kj.
 * z, out: fp32 [B, N, N, c_z]; mask: fp32 [B, N, N] or NULL. */
GTK_API int gtk_trimul_forward(int outgoing, const float* z, const float* mask, const void* packed, float* out,
                       int add_residual, void* workspace, size_t workspace_bytes, int64_t B, int64_t N, int c_z,
                       int c_hidden, uint32_t* status, void* stream);

/* gtk_trimul_forward without a workspace argument, for callers that cannot allocate
 * device memory: plugin hosts that own every device allocation and give their plugins no
 * allocator, serving processes that run under a fixed memory budget, and latency paths
 * that must not call cudaMalloc (it can synchronise the device). The library brings its
 * own scratch: a 24 MiB array in device memory, created on every GPU that loads the
 * library and kept until the process exits. It covers B * N * round_up(N, 8) <= 32768
 * (for example B = 1, N <= 176, or B = 2, N = 128); larger sizes return
 * GTK_ERR_WORKSPACE with a message naming the limit. Nothing in the scratch needs to
 * start at zero: every byte a call reads was written earlier in the same call.
 * The first call on a device looks up the scratch address on that device (the device
 * must be current); make that first call before any stream capture. That address is kept
 * for the life of the process, so after a cudaDeviceReset of a device this entry point
 * must not be called on that device again in the same process. All calls share the
 * one array, so calls whose work overlaps on the GPU (different streams, or different
 * host threads without ordering) race on it: serialise them.
 * No counterpart in the reference (its `_C` functions allocate their outputs). */
GTK_API int gtk_trimul_forward_noalloc(int outgoing, const float* z, const float* mask, const void* packed,
                                       float* out, int add_residual, int64_t B, int64_t N, int c_z, int c_hidden,
                                       uint32_t* status, void* stream);

/* Stage entry points (used by tests and by the multi-GPU driver).
 *
 * Plane buffers hold one fp16 N-wide row per (pair row, channel):
 *   X[b][r][c][col], element offset ((b*R + r)*C + c)*ld + col,
 * with the pitch `ld` (elements) a multiple of 8 and >= the column count.
 * gtk_plane_pitch(N) gives the pitch the forward entry points use. */
GTK_API int64_t gtk_plane_pitch(int64_t N);

/* LN_in + gated projections + mask for `rows` pair rows of z ([B, rows, N, c_z]);
 * writes a and b planes [B, rows, c, ld]. mask: [B, rows, N] or NULL. */
GTK_API int gtk_trimul_project(const float* z, const float* mask, const void* packed, void* a_planes, void* b_planes,
                       int64_t ld, int64_t B, int64_t rows, int64_t N, uint32_t* status, void* stream);
/* As gtk_trimul_project, for one shard of `rows` pair rows that starts at row `row0` of a
 * row-sharded pair tensor with `dst_rows` rows in all: channel c of the a (b) planes is
 * written to a_dsts[c / (128/P)] (b_dsts[...]), a [B][dst_rows][128/P][ld] channel shard,
 * at its rows row0.., so each channel group lands directly in the buffer of the rank that
 * contracts it (host arrays of P <= 8 device addresses; peer GPUs' buffers mapped into this
 * process are allowed). */
GTK_API int gtk_trimul_project_sharded(const float* z, const float* mask, const void* packed, void* const* a_dsts,
                                       void* const* b_dsts, int P, int64_t dst_rows, int64_t row0, int64_t ld,
                                       int64_t B, int64_t rows, int64_t N, uint32_t* status, void* stream);

/* Per-channel contraction on plane buffers, for every (b, c):
 *  outgoing: x[b][i][c][j] = sum_k a[b][i][c][k] * bb[b][j][c][k]  (a: [B,M,C,lda], bb: [B,Nj,C,ldb])
 *  incoming: x[b][i][c][j] = sum_k a[b][k][c][i] * bb[b][k][c][j]  (a: [B,K,C,lda], bb: [B,K,C,ldb])
 * x: [B, M, C, ldx] holds the fp32 sums times out_scale, rounded to fp16 (saturating);
 * the forward path uses out_scale = 1/K. i < M, j < Nj, k < K. */
GTK_API int gtk_trimul_contract(int outgoing, const void* a_planes, const void* b_planes, void* x_planes,
                                int64_t B, int64_t C, int64_t M, int64_t Nj, int64_t K, int64_t lda, int64_t ldb,
                                int64_t ldx, float out_scale, uint32_t* status, void* stream);

/* LN_out + linear_z + output gate (+ residual) for `rows` pair rows:
 * out[b,r,j,:] = gate(z[b,r,j]) * linear_z(LN_out(x[b][r][:][j] / x_scale)) (+ z[b,r,j] if add_residual);
 * x_scale is the out_scale the x planes were written with. */
GTK_API int gtk_trimul_finish(const float* z, const void* x_planes, int64_t ldx, float x_scale, const void* packed,
                              float* out, int add_residual, int64_t B, int64_t rows, int64_t N, uint32_t* status,
                              void* stream);

/* ---------------------------------------------------------------------------------
 * Triangle attention around the starting / ending node (Algorithms 13/14).
 * Replaces `_C.triangle_attention_starting` / `_C.triangle_attention_ending`
 * (kernels/bindings.cpp:30-46, bound at :82-90) together with the PyTorch code of
 * `TriangleAttention._forward_cuda` (src/genie_tk/triangle_attention.py:145-179), which
 * in the reference always falls back to `_forward_pytorch` (:100-143): LN, triangle bias,
 * mask bias inf*(mask-1), gated 4-head attention, linear_o. The ending node is computed
 * on z^T through transposed descriptors; the result is in z's orientation.
 * ------------------------------------------------------------------------------- */

/* fp32 device pointers to the parameters of a reference TriangleAttention
 * (src/genie_tk/triangle_attention.py:70-82, src/genie_tk/primitives.py:319-328). */
typedef struct gtk_triatt_params {
  const float* ln_w;   /* layer_norm.weight [c_in] */
  const float* ln_b;   /* layer_norm.bias [c_in] */
  const float* bias_w; /* linear.weight [heads, c_in] (triangle bias, no bias term) */
  const float* q_w;    /* mha.linear_q.weight [c_hidden, c_in] */
  const float* k_w;    /* mha.linear_k.weight */
  const float* v_w;    /* mha.linear_v.weight */
  const float* g_w;    /* mha.linear_g.weight [c_hidden, c_in] */
  const float* g_b;    /* mha.linear_g.bias [c_hidden] */
  const float* o_w;    /* mha.linear_o.weight [c_in, c_hidden] */
  const float* o_b;    /* mha.linear_o.bias [c_in] */
} gtk_triatt_params;

GTK_API size_t gtk_triatt_packed_bytes(int c_in, int c_hidden, int heads);
GTK_API int gtk_triatt_pack(const gtk_triatt_params* params, int c_in, int c_hidden, int heads, void* packed,
                            size_t packed_bytes, void* stream);
GTK_API size_t gtk_triatt_workspace_bytes(int64_t B, int64_t N, int c_in, int c_hidden, int heads);

/* out = update(z) or z + update(z) (add_residual; out may equal z). `inf` is the module's
 * mask constant (1e9 in the reference). z, out fp32 [B, N, N, c_in]; mask fp32 [B, N, N] or
 * NULL. */
GTK_API int gtk_triatt_forward(int starting, const float* z, const float* mask, const void* packed, float* out,
                               int add_residual, void* workspace, size_t workspace_bytes, int64_t B, int64_t N,
                               int c_in, int c_hidden, int heads, float inf, uint32_t* status, void* stream);

/* Stage entry points over a workspace, for `rows` problem rows starting at global row `row0`
 * (rows = N, row0 = 0 for a whole pair tensor; a shard of a row-sharded pair tensor
 * otherwise, starting orientation only: a row-sharded caller runs the ending node as the
 * starting node of the transposed shards). offsets[7] receives the byte offsets of
 *   q, k, v  [B*rows][H][N][32] fp16 (q scaled by log2(e)/sqrt(32)),
 *   g        [B*rows*N][128] fp16 (sigmoid applied),
 *   og       [B*rows*N][128] fp16 (gated attention output),
 *   bias     [N][B][H][round_up(N,8)] bf16 (the triangle bias, log2 units, ALL N rows:
 *            project writes rows row0..row0+rows-1; the core reads every row, so a
 *            row-sharded caller all-gathers this region in place between the two),
 * and offsets[6] the workspace size in bytes. All in the orientation of the problem
 * (z^T for the ending node). */
GTK_API int gtk_triatt_workspace_offsets(int64_t B, int64_t rows, int64_t N, int64_t* offsets);
/* z: the shard's rows [B, rows, N, 128] fp32. */
GTK_API int gtk_triatt_project(int starting, const float* z, const void* packed, void* workspace, int64_t B,
                               int64_t rows, int64_t N, int64_t row0, uint32_t* status, void* stream);
/* mask: the WHOLE problem's [B, N, N] fp32 (or NULL); the shard's rows start at row0. */
GTK_API int gtk_triatt_core(int starting, const float* mask, void* workspace, int64_t B, int64_t rows, int64_t N,
                            int64_t row0, float inf, uint32_t* status, void* stream);
/* z, out: the shard's rows [B, rows, N, 128] fp32. */
GTK_API int gtk_triatt_finish(int starting, const float* z, const void* packed, void* workspace, float* out,
                              int add_residual, int64_t B, int64_t rows, int64_t N, uint32_t* status, void* stream);

/* ---------------------------------------------------------------------------------
 * Data movement for the row-sharded stack (one process per GPU; the pair tensor is split
 * over its first pair index into P shards of R = N / P rows). The reference has no
 * multi-GPU path; these serve the host driver that exchanges shards with NCCL
 * (all-to-alls between row shards and channel shards of the multiplicative update's
 * planes, an all-gather of the triangle-bias rows, all-to-all transposes of the pair
 * tensor for the ending-node attention).
 * ------------------------------------------------------------------------------- */

/* `height` rows of `width` bytes from src (row pitch spitch) to dst (row pitch dpitch).
 * Width, pitches and both pointers must be multiples of 16 bytes. */
GTK_API int gtk_copy_2d(void* dst, int64_t dpitch, const void* src, int64_t spitch, int64_t width, int64_t height,
                        void* stream);
/* The same 2D copy on the GPU's copy engines (cudaMemcpy2DAsync on `stream`) instead of
 * a kernel: no SM time. dst may be a peer GPU's memory mapped into this process (CUDA
 * IPC); the copy is stream-ordered like a kernel. */
GTK_API int gtk_copy_2d_dma(void* dst, int64_t dpitch, const void* src, int64_t spitch, int64_t width, int64_t height,
                            void* stream);
/* `depth` slabs of the 2D copy above; slab k starts at dst + k*dslab and src + k*sslab
 * (slab strides are multiples of 16 bytes as well). */
GTK_API int gtk_copy_3d(void* dst, int64_t dpitch, int64_t dslab, const void* src, int64_t spitch, int64_t sslab,
                        int64_t width, int64_t height, int64_t depth, void* stream);

/* Per-peer chunks of a pair-grid transpose: for src [B][R][C][128] fp32,
 * dst[q][b][x][y][:] = src[b][y][q*(C/P) + x][:]  (q < P, x < C/P, y < R).
 * Chunk q (B*(C/P)*R pair vectors) is what peer q receives in an all-to-all; peer q then
 * places the chunk from peer p at pair-column offset p*R of its transposed shard. */
GTK_API int gtk_pair_transpose_pack(const float* src, float* dst, int64_t B, int64_t R, int64_t C, int64_t P,
                                    void* stream);

/* Peer-memory exchange (one process per GPU on one NVLink/NVSwitch node). Buffers that
 * other ranks write into are allocated here and shared by CUDA IPC handles; the push
 * kernels write each peer's share straight into that peer's buffer (packing, transfer
 * and placement in one pass), and gtk_peer_barrier orders the pushes across ranks on the
 * stream. No multicast object and no cluster multicast is involved: plain stores to
 * peer memory over NVLink. */
#define GTK_PEER_HANDLE_BYTES 64
/* cudaMalloc + zero fill + IPC handle (GTK_PEER_HANDLE_BYTES bytes written to `handle`). */
GTK_API int gtk_peer_alloc(size_t bytes, void** ptr, void* handle);
GTK_API int gtk_peer_free(void* ptr);
/* Map a peer's buffer (from its handle) into this process; gtk_peer_close unmaps it. */
GTK_API int gtk_peer_open(const void* handle, void** ptr);
GTK_API int gtk_peer_close(void* ptr);
/* Slab k (k < P) of `height` rows of `width` bytes at src + k*sslab (row pitch spitch) is
 * written to dsts[k] + doff (row pitch dpitch). dsts: device array of P base addresses.
 * All sizes, offsets and addresses are multiples of 16 bytes. */
GTK_API int gtk_push_3d(const uint64_t* dsts, int P, int64_t doff, int64_t dpitch, const void* src, int64_t spitch,
                        int64_t sslab, int64_t width, int64_t height, void* stream);
/* Pair (b, y, q*(C/P) + x) of src [B][R][C][128] fp32 is written to peer q's transposed
 * shard dsts[q] [B][C/P][ndst][128] at (b, x, row0 + y). */
GTK_API int gtk_push_pair_transpose(const float* src, const uint64_t* dsts, int64_t B, int64_t R, int64_t C,
                                    int64_t P, int64_t ndst, int64_t row0, void* stream);
/* The channel-sharded contraction of a row-sharded stack with its scatter back to the row
 * owners fused into its stores: x tiles of the C channels computed here (over all M rows) are
 * TMA-stored into the owner of their rows, p = row / (M/P), as channels c_off .. c_off+C-1 of
 * p's x planes [B][M/P][C_dst][ld_dst] (fp16, scaled by out_scale as gtk_trimul_contract).
 * dst_bases: HOST array of the P ranks' x-plane addresses; M/P a multiple of 128, P <= 8.
 * Replaces gtk_trimul_contract + the x push of the sharded stack (no reference counterpart). */
GTK_API int gtk_trimul_contract_to_peers(int outgoing, const void* a_planes, const void* b_planes,
                                         const uint64_t* dst_bases, int P, int64_t B, int64_t C, int64_t M,
                                         int64_t Nj, int64_t K, int64_t lda, int64_t ldb, int64_t C_dst,
                                         int64_t c_off, int64_t ld_dst, float out_scale, uint32_t* status,
                                         void* stream);
/* K4e of a row shard with the pair-grid transpose fused into its stores: the finished
 * update out = z + og W_o^T + b_o (+ z when add_residual) of the starting-orientation shard
 * (rows local rows from global row row0, the workspace of gtk_triatt_core) is written
 * straight into the P ranks' transposed shards, pair (b, y, j) to rank q = j / rows at
 * (b, j - q*rows, row0 + y), by TMA stores into the peers' memory. dst_bases: HOST array of
 * the P shards' device addresses ([B][rows][N][128] fp32 each, 16-byte aligned); rows * P
 * = N, rows a multiple of 128, P <= 8. Replaces gtk_triatt_finish + gtk_push_pair_transpose
 * in the sharded stack (no reference counterpart: the reference runs on one device). */
GTK_API int gtk_triatt_finish_to_peers(const float* z, const void* packed, void* workspace,
                                       const uint64_t* dst_bases, int P, int64_t B, int64_t rows, int64_t N,
                                       int64_t row0, int add_residual, uint32_t* status, void* stream);
/* Barrier over P ranks: each rank publishes `epoch` into every rank's flag array (P uint32
 * each, zero-initialised peer memory; flag_ptrs: device array of the P arrays' addresses)
 * and waits until all P have published it. Stream-ordered: pushes enqueued before it on
 * every rank are visible to work enqueued after it. Bounded: after 2 s the status word
 * gets GTK_STATUS_TIMEOUT_PEER. Epochs must increase by one per barrier. */
GTK_API int gtk_peer_barrier(const uint64_t* flag_ptrs, int rank, int P, uint32_t epoch, uint32_t* status,
                             void* stream);

/* ---------------------------------------------------------------------------------
 * Pair transition (reference src/genie_tk/pair_transform.py:64-84, the feed-forward of
 * PairTransformLayer; no counterpart in kernels/bindings.cpp) with the layer's residual and
 * final mask multiply (pair_transform.py:190-193) folded in. c_p = 128 with n <= 4 runs on
 * the tuned kernels (a narrower hidden layer zero-padded to 512 units); other widths (c_p
 * <= 512, hidden n c_p <= 2048) on the general-shape kernels.
 * ------------------------------------------------------------------------------- */
typedef struct gtk_transition_params {
  const float* ln_w; /* layer_norm.weight [c_p] */
  const float* ln_b; /* layer_norm.bias [c_p] */
  const float* w1;   /* linear_1.weight [n c_p, c_p] */
  const float* b1;   /* linear_1.bias [n c_p] (NULL = zero) */
  const float* w2;   /* linear_2.weight [c_p, n c_p] */
  const float* b2;   /* linear_2.bias [c_p] (NULL = zero) */
} gtk_transition_params;

GTK_API size_t gtk_transition_packed_bytes(int c_p, int n);
GTK_API int gtk_transition_pack(const gtk_transition_params* params, int c_p, int n, void* packed,
                                size_t packed_bytes, void* stream);
/* Workspace for the hidden rows (fp16). */
GTK_API size_t gtk_transition_workspace_bytes(int64_t B, int64_t N, int c_p, int n);
/* out = (add_residual ? z : 0) + transition(z), then times mask[b, i, j] when mask is not
 * NULL. z, out fp32 [B, N, N, c_p] (out may equal z); mask fp32 [B, N, N] or NULL. */
GTK_API int gtk_transition_forward(const float* z, const float* mask, const void* packed, float* out,
                                   int add_residual, void* workspace, size_t workspace_bytes, int64_t B, int64_t N,
                                   int c_p, int n, uint32_t* status, void* stream);

/* ---------------------------------------------------------------------------------
 * Pair embedding producer (reference examples/basic_usage.py:181-199; no counterpart in
 * kernels/bindings.cpp): p[b,i,j] = weight @ [s[b,i]; s[b,j]] + bias (nn.Linear(2 c_s, c_p)
 * on the concatenation, never formed) and p_mask[b,i,j] = mask[b,i] * mask[b,j], written
 * into the fp32 pair layout [B, rows, N, c_p] for rows row0 .. row0+rows-1 (all of them:
 * rows = N, row0 = 0; a row shard otherwise). c_p in 1..4096; out 16-byte aligned when c_p
 * is a multiple of 4 (4-byte aligned otherwise).
 * s fp32 [B, N, c_s]; mask fp32 [B, N] or NULL; weight fp32 [c_p, 2 c_s]; bias [c_p] or
 * NULL; pair_mask fp32 [B, rows, N] or NULL (not written).
 * ------------------------------------------------------------------------------- */
GTK_API size_t gtk_pair_embed_workspace_bytes(int64_t B, int64_t N, int c_p);
GTK_API int gtk_pair_embed(const float* s, const float* mask, const float* weight, const float* bias, float* out,
                           float* pair_mask, void* workspace, size_t workspace_bytes, int64_t B, int64_t N,
                           int64_t rows, int64_t row0, int c_s, int c_p, void* stream);

/* ---------------------------------------------------------------------------------
 * Training-mode channel dropout of the residual updates (reference
 * src/genie_tk/pair_transform.py:26-61, applied at :182-189 as p = p + dropout(update)).
 * DropoutRowwise draws one mask [B, 1, N, C] shared by every row i (it varies with the
 * column j); DropoutColumnwise one mask [B, N, 1, C] shared by every column j (it varies
 * with the row i). Here a mask is a keep-bit array of B * N vectors of G = ceil(C / 128)
 * groups of 128 bits: vector (b, t) is the 4 G uint32 words at (b * N + t) * 4 G, and
 * channel c is kept when bit c % 32 of word c / 32 of it is set. (For C <= 128 that is four
 * words per vector; the generator and the packer below make 128-bit groups, so a C-channel
 * mask is n_vectors = B * N * G of them.) Kept channels are multiplied by `scale`
 * (1 / (1 - p)); dropped ones add nothing. The *_forward_dropout entry points apply the
 * mask inside the residual epilogue: out = z + keep * scale * update (add_residual = 1) or
 * out = keep * scale * update (add_residual = 0).
 * ------------------------------------------------------------------------------- */
typedef struct gtk_dropout {
  const uint32_t* keep_bits; /* device, 16-byte aligned, B * N * 4 * ceil(C / 128) words */
  float scale;               /* multiplier of the kept channels: finite, >= 0 */
  int shared_across_rows;    /* 1: DropoutRowwise (vector t = j); 0: DropoutColumnwise (t = i) */
} gtk_dropout;

/* Keep bits for n_vectors vectors from the counter-based generator Philox4x32-10 (Salmon,
 * Moraes, Dror, Shaw, SC'11): channel c of vector v is kept when output word c % 4 of
 * Philox(counter = {lo32(v*32 + c/4), hi32(v*32 + c/4), lo32(offset), hi32(offset)},
 * key = {lo32(seed), hi32(seed)}) is >= floor(p * 2^32). 0 <= p < 1. Advance `offset`
 * between draws of one seed. No counterpart in the reference (it draws with nn.Dropout). */
GTK_API int gtk_dropout_keep_bits_philox(uint64_t seed, uint64_t offset, double p, int64_t n_vectors,
                                         uint32_t* keep_bits, void* stream);

/* Keep bits from a multiplier tensor fp32 [n_vectors][128] whose dropped channels are 0
 * (the reference's own mask, nn.Dropout applied to ones, packed). */
GTK_API int gtk_dropout_pack_keep_bits(const float* multipliers, int64_t n_vectors, uint32_t* keep_bits,
                                       void* stream);

/* gtk_trimul_forward / gtk_triatt_forward with the dropout applied to the update before
 * the residual add; dropout = NULL is the plain entry point. */
GTK_API int gtk_trimul_forward_dropout(int outgoing, const float* z, const float* mask, const void* packed,
                                       float* out, int add_residual, const gtk_dropout* dropout, void* workspace,
                                       size_t workspace_bytes, int64_t B, int64_t N, int c_z, int c_hidden,
                                       uint32_t* status, void* stream);
GTK_API int gtk_triatt_forward_dropout(int starting, const float* z, const float* mask, const void* packed,
                                       float* out, int add_residual, const gtk_dropout* dropout, void* workspace,
                                       size_t workspace_bytes, int64_t B, int64_t N, int c_in, int c_hidden,
                                       int heads, float inf, uint32_t* status, void* stream);

/* ---------------------------------------------------------------------------------
 * The attention core for training (the gradient the reference gets from PyTorch autograd
 * through src/genie_tk/primitives.py:134-164 and triangle_attention.py:115-137), in the
 * block's frame (z for the starting node, z^T for the ending node), pair row i, query j,
 * key k, head h of head_dim d:
 *   s = q[i,j,h] . k[i,k,h] / sqrt(d) + inf (mask[i,k] - 1) + tri[h,j,k],
 *   o[i,j,h] = sum_k softmax_k(s) v[i,k,h].
 * The kernels never form the [B, N, heads, N, N] scores: 64-row tiles of fp16 operand planes
 * are copied into shared memory (double buffered) and every product runs on the tensor cores
 * (mma.sync m16n8k16, fp32 accumulation); scale, bias, mask and softmax are fp32.
 * Operand planes (written by the two pack entry points, 16-byte aligned):
 *   q, k, v, dO: fp16 [B, N(i), heads, N(j), Dp], Dp = head_dim rounded up to 16, 32 or 64
 *                (zero-padded), gtk_attn_core_packed_bytes(B, N, heads, head_dim) bytes each;
 *   tri:         fp16 [B, heads, N(j), Np], Np = N rounded up to a multiple of 8,
 *                gtk_attn_core_bias_bytes(B, N, heads) bytes.
 * mask: fp32 [B, N(i), N(k)] in the block's frame, or NULL. o, dq, dk, dv: fp32
 * [B, N(i), N(j), heads * head_dim] (the projections' layout); dtri fp32 [B, heads, N, N];
 * stats 8-byte aligned. head_dim <= 64.
 * ------------------------------------------------------------------------------- */
GTK_API size_t gtk_attn_core_packed_bytes(int64_t B, int64_t N, int heads, int head_dim);
GTK_API size_t gtk_attn_core_bias_bytes(int64_t B, int64_t N, int heads);
/* fp32 [B, N, N, heads * head_dim] -> an fp16 operand plane, times `scale`. */
GTK_API int gtk_attn_core_pack(const float* src, int64_t B, int64_t N, int heads, int head_dim, float scale,
                               void* dst, void* stream);
/* fp32 tri [B, heads, N, N] -> its fp16 plane. */
GTK_API int gtk_attn_core_pack_bias(const float* tri, int64_t B, int64_t N, int heads, void* dst, void* stream);

/* o and the softmax statistics: stats[b][i][h][j] = (max of the base-2 scores, 1 / sum of
 * 2^(score - max)), two floats. q, k, v packed with scale 1. */
GTK_API int gtk_attn_core_forward(const void* q, const void* k, const void* v, const void* tri,
                                  const float* mask, int64_t B, int64_t N, int heads, int head_dim, float inf,
                                  float* o, float* stats, void* stream);
/* dq, dk, dv and dtri from the output gradient, the forward's stats and
 * dsum[b][i][h][j] = sum_e dO o (over the head's d channels, fp32, unscaled). dO is packed
 * times dO_scale (> 0; a power of two near 1 / max|dO| keeps gradients of any magnitude at
 * 11 bits); the results are divided by it again. dtri sums the score gradients over the rows i. */
GTK_API int gtk_attn_core_backward(const void* q, const void* k, const void* v, const void* tri,
                                   const float* mask, const float* stats, const void* dO, const float* dsum,
                                   float dO_scale, int64_t B, int64_t N, int heads, int head_dim, float inf,
                                   float* dq, float* dk, float* dv, float* dtri, void* stream);

/* ---------------------------------------------------------------------------------
 * The generic multi-head attention core of the reference's `Attention` module
 * (src/genie_tk/primitives.py:114-178, between its projections and its gate):
 *   o[l, q, h, :] = sum_k softmax_k(scale q[l,q,h] . k[l,k,h] + bias0 + bias1) v[l, k, h, :]
 * q, o fp32 [L0 * L1, Q, heads * head_dim]; k, v fp32 [L0 * L1, K, heads * head_dim];
 * head_dim <= 64. Each bias is optional (NULL) and read through five element strides
 * strides[0..4] over (l0, l1, h, q, k), l = l0 * L1 + l1: a zero stride broadcasts, so the
 * reference's mask bias [*, 1, 1, K] and pair bias [*, H, Q, K] are read in place. A row
 * whose scores are all -inf gives NaN, as softmax does. Same arithmetic as the core above.
 * ------------------------------------------------------------------------------- */
GTK_API int gtk_mha_forward(const float* q, const float* k, const float* v, const float* bias0,
                            const int64_t* strides0, const float* bias1, const int64_t* strides1, int64_t L0,
                            int64_t L1, int64_t Q, int64_t K, int heads, int head_dim, float scale, float* o,
                            void* stream);

/* ---------------------------------------------------------------------------------
 * LayerNorm over the last axis: the reference's `_C.layernorm(x, gamma, beta, eps)`
 * (kernels/bindings.cpp:93-95; host code kernels/fused_layernorm/layernorm.cu:17-44).
 * x, out fp32 [rows, D] (out may equal x); gamma, beta fp32 [D]; biased variance.
 * ------------------------------------------------------------------------------- */
GTK_API int gtk_layernorm(const float* x, const float* gamma, const float* beta, float* out, int64_t rows,
                          int64_t D, float eps, void* stream);

/* The reference's `_C.fused_layernorm_linear(x, gamma, beta, weight, bias, eps)`
 * (kernels/bindings.cpp:97-101; layernorm.cu:46-76): out = LayerNorm(x) weight^T + bias in
 * one kernel -- each CTA normalises its 64 rows while loading them, so the normalised rows
 * never reach memory. x fp32 [rows, D_in]; weight fp32 [D_out, D_in] (nn.Linear's layout:
 * the reference's [D_in, D_out] operand transposed); bias fp32 [D_out] or NULL; out fp32
 * [rows, D_out]; out must not alias x. fp32 CUDA-core arithmetic. */
GTK_API int gtk_layernorm_linear(const float* x, const float* gamma, const float* beta, const float* weight,
                                 const float* bias, float* out, int64_t rows, int64_t D_in, int64_t D_out, float eps,
                                 void* stream);

/* out = (x * sigmoid(gate) if gate else x) weight^T + bias: the projections of the
 * reference's Linear / Attention modules (primitives.py:43-62, :124-178). x, gate fp32
 * [rows, D_in] (gate may be NULL); weight fp32 [D_out, D_in]; bias fp32 [D_out] or NULL;
 * out fp32 [rows, D_out], aliasing neither x nor gate. fp32 CUDA-core arithmetic. */
GTK_API int gtk_linear(const float* x, const float* gate, const float* weight, const float* bias, float* out,
                       int64_t rows, int64_t D_in, int64_t D_out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GENIE_TK_B200_H_ */
