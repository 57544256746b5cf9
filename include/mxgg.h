/*
 * mxgg -- Blackwell (sm_100a) MXFP8 grouped-GEMM library, C ABI.
 *
 * Drop-in replacement for the hot path of indianspeedster/grouped-gemms:
 * the two grouped-GEMM entry points and the MX quantiser.  Every function
 * takes plain device pointers, element counts and a CUDA stream passed as
 * `void*` (a cudaStream_t / CUstream; NULL = legacy default stream), enqueues
 * its work on that stream, never synchronises and never allocates: scratch
 * memory a call needs is passed in by the caller (see *_workspace_size).
 * All functions return MXGG_OK (0) or an error code; mxgg_last_error()
 * returns a message for the calling thread's last failure.
 *
 * Data formats (as produced by the reference's utils.to_mx, utils.py:67-105):
 *   - element data: float8_e4m3fn bytes, row-major, quantised along the
 *     contiguous (contraction) dimension;
 *   - scales: e8m0 bytes (uint8 or float8_e8m0fnu), one per 32 contiguous
 *     elements, row-major (rows, contraction / 32);
 *   - group_end_offsets: int32 cumulative group ends (E,), device memory.
 */
#ifndef MXGG_H_
#define MXGG_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define MXGG_OK 0
#define MXGG_ERR_INVALID 1     /* bad argument: shape, alignment, null pointer */
#define MXGG_ERR_CUDA 2        /* a CUDA runtime/driver call failed */
#define MXGG_ERR_UNSUPPORTED 3 /* valid request outside what this build handles */

/* element types for inputs / outputs */
#define MXGG_DTYPE_BF16 0
#define MXGG_DTYPE_F16 1
#define MXGG_DTYPE_F32 2

/* quantiser modes */
#define MXGG_QUANT_ROWS 0 /* blocks along the contiguous last dim (reference to_mx) */
#define MXGG_QUANT_COLS 1 /* blocks along the leading dim, output transposed */

/* scale layouts */
#define MXGG_SCALE_ROW_MAJOR 0 /* (rows, cols/32), the reference layout */
#define MXGG_SCALE_BLOCKED 1   /* 128x4 atoms (rows padded to 128, cols/32 to 4) */
/*
 * The blocked scale layout the grouped GEMMs read (torch's layout for its
 * grouped MXFP8 GEMMs).  A scale matrix of R rows and C/32 columns (C the
 * contraction) is stored as 512-byte atoms [slab][ceil(C/128)][512 B], one
 * slab per 128 rows, byte (r % 32) * 16 + ((r % 128) / 32) * 4 + k % 4 of
 * atom (slab, k / 4) holding row r, k-block k of the slab.  Rows are cut into
 * segments and every segment starts a new slab:
 *   forward / dgrad A   segments = the groups (group_end_offsets)
 *   forward / dgrad B   segments = the experts (N rows each)
 *   wgrad A and B       one segment (the whole operand: MXGG_SCALE_BLOCKED)
 * mxgg_quantize_mx_blocked writes the segmented form, mxgg_quantize_mx with
 * MXGG_SCALE_BLOCKED the one-segment form.  Padding (rows past a segment's
 * end in its last slab, k-blocks past C/32) feeds no stored output. */

/* element formats of a GEMM operand */
#define MXGG_FMT_E4M3 0 /* MXFP8: one e4m3 byte per element */
#define MXGG_FMT_E2M1 1 /* MXFP4: two e2m1 values per byte, element 2i in the low nibble */

/*
 * Per-call kernel configuration for the *_cfg entry points (no counterpart in
 * the reference, whose Triton wrappers take BLOCK_* / GROUP_M keywords per
 * call, forward.py:461-484).  A field left 0 takes the process default set
 * by mxgg_set_tile_config / mxgg_set_schedule, and those default to the
 * library's own choice.  The struct is read during the call only; two
 * threads may issue differently configured GEMMs concurrently.
 *   tile_m     128: one CTA per output tile; 256: a CTA pair (cta_group::2)
 *   tile_n     128 or 256 output columns per tile
 *   group_m    rasterisation band, in row tiles (>= 1)
 *   schedule   MXGG_SCHED_TILES or MXGG_SCHED_SPLIT_TAIL (see mxgg_set_schedule)
 *   split_max  most pieces per split tile (2..64)
 *   scale_layout  MXGG_SCALE_ROW_MAJOR (0): a_scale / b_scale are the
 *              reference's row-major e8m0 matrices, re-laid into the
 *              workspace by a pack launch before the GEMM.
 *              MXGG_SCALE_BLOCKED: they are already in the blocked layout
 *              (see MXGG_SCALE_BLOCKED; 16-byte aligned, A at least the sum
 *              over groups of ceil(rows_g / 128) slabs -- at most
 *              mxgg_blocked_scale_bytes(M, K, E) bytes -- B n_experts *
 *              ceil(N / 128) slabs); the GEMM reads them in place and
 *              launches nothing else.  Results are bit-identical.
 *              Forward, dgrad and wgrad entry points; not the expert-parallel
 *              one.
 *   reserved   must be zero
 */
typedef struct mxgg_gemm_config {
  int32_t tile_m;
  int32_t tile_n;
  int32_t group_m;
  int32_t schedule;
  int32_t split_max;
  int32_t scale_layout;
  int32_t reserved[2];
} mxgg_gemm_config;

/*
 * Scratch ("workspace") for one grouped-GEMM call: the row-major scales are
 * re-laid into the 128x4 atoms the tensor cores read, one atom per 128-row
 * slab and 128-element contraction stage (the reference re-lays its scales on
 * every call too, forward.py:537-561).  Returns the bytes to pass as
 * `workspace_bytes` (256-byte aligned device memory), or -1 for bad sizes.
 * The workspace is scratch: its contents need not survive between calls, and
 * calls that run concurrently need separate workspaces.
 */
int64_t mxgg_grouped_mm_workspace_size(int64_t M, int64_t N, int64_t K, int64_t E);
int64_t mxgg_wgrad_workspace_size(int64_t N, int64_t K, int64_t M, int64_t E);

/*
 * Forward / dgrad grouped GEMM: out[rows of group g] = A[rows] @ B[g]^T.
 * Replaces triton_mxfp8_grouped_mm (reference kernels/forward.py:461-606).
 *   a        (M, K) e4m3            a_scale (M, K/32) e8m0
 *   b        (E, N, K) e4m3         b_scale (E, N, K/32) e8m0
 *   group_end_offsets (E,) int32, device; group g owns rows
 *            [offs[g-1], offs[g]) (offs[-1] := 0).  Any row boundaries work.
 *   out      (M, N) of out_dtype (MXGG_DTYPE_BF16/F16/F32).  Rows at or past
 *            offs[E-1] are not written (forward.py:583 leaves them unset).
 *   workspace  >= mxgg_grouped_mm_workspace_size(M, N, K, E) bytes.
 * Requirements: K % 32 == 0; a, b 16-byte aligned; 1 <= E <= 256.
 */
int mxgg_grouped_mm(const void* a, const void* b, const void* a_scale, const void* b_scale,
                    const int32_t* group_end_offsets, int64_t M, int64_t N, int64_t K, int64_t E,
                    void* out, int out_dtype, void* workspace, int64_t workspace_bytes, void* stream);
/* mxgg_grouped_mm with its own tile and schedule choice (config may be null:
 * the process defaults).  The same workspace size serves every config. */
int mxgg_grouped_mm_cfg(const void* a, const void* b, const void* a_scale, const void* b_scale,
                        const int32_t* group_end_offsets, int64_t M, int64_t N, int64_t K, int64_t E, void* out,
                        int out_dtype, const mxgg_gemm_config* config, void* workspace, int64_t workspace_bytes,
                        void* stream);

/*
 * Forward / dgrad grouped GEMM that allocates nothing and takes no workspace.
 * No counterpart in the reference: it exists for callers that cannot get
 * device memory at call time -- code running where the allocator must not be
 * entered (a runtime that reserved all device memory up front, an inference
 * server or plugin host that forbids allocation after start-up, a
 * latency-critical loop that must not risk cudaMalloc's implicit device
 * synchronisation) and that cannot hold a workspace of its own.
 * Same arguments and results as mxgg_grouped_mm minus the workspace.  Its
 * scratch is one fixed 32 MiB array in device memory that every GPU loading
 * this library keeps until the process exits.  The array holds the packed
 * scale atoms first: a problem whose packed scales alone exceed 32 MiB is
 * rejected with MXGG_ERR_UNSUPPORTED.  The split-tail schedule's partial
 * tiles (about 21 MB) go after them when they fit; when they do not (for
 * example E=8, M=16640, N=K=8192), the call deals every tile whole
 * (MXGG_SCHED_TILES), so its result equals mxgg_grouped_mm run with that
 * schedule, and may differ from the split-tail result in the last bits of
 * the fp32 sums.  The first call on a device resolves the array's
 * address on that device (the device must be current); make that first call
 * before any stream capture.  All calls share the array, which keeps the last
 * call's contents (nothing in it needs to start zeroed: each call rewrites
 * what it reads): calls whose work overlaps on the GPU, e.g. on two streams,
 * race on it and must be serialised by the caller.
 */
int mxgg_grouped_mm_noalloc(const void* a, const void* b, const void* a_scale, const void* b_scale,
                            const int32_t* group_end_offsets, int64_t M, int64_t N, int64_t K, int64_t E,
                            void* out, int out_dtype, void* stream);

/*
 * Forward grouped GEMM over segments that share experts: segment s (rows
 * [segment_end_offsets[s-1], segment_end_offsets[s]) of A) is multiplied by
 * B[segment_expert[s]].  This is the layout an expert-parallel all-to-all
 * delivers (rows grouped by source rank, then by expert), so the GEMM reads
 * the receive buffer as it lands.  No counterpart in the reference.
 *   b        (n_experts, N, K) e4m3,   b_scale (n_experts, N, K/32)
 *   segment_end_offsets (n_segments,) int32, device, cumulative
 *   segment_expert      (n_segments,) int32, device, in [0, n_experts)
 *   b_format  MXGG_FMT_E4M3, or MXGG_FMT_E2M1 for MXFP4 weights: b holds
 *             (n_experts, N, K/2) bytes, two e2m1 values per byte (element
 *             2i in the low nibble), 32-byte aligned, K % 128 == 0; the
 *             scales are still one e8m0 per 32 elements.  MXFP4 x MXFP8 runs
 *             on the same kind::mxf8f6f4 tensor-core path (no reference
 *             counterpart: its kernels are MXFP8 only).
 * Other arguments as mxgg_grouped_mm; the workspace is at least
 * mxgg_grouped_mm_segments_workspace_size(M, N, K, n_segments, n_experts).
 */
int64_t mxgg_grouped_mm_segments_workspace_size(int64_t M, int64_t N, int64_t K, int64_t n_segments,
                                                int64_t n_experts);
int mxgg_grouped_mm_segments(const void* a, const void* b, const void* a_scale, const void* b_scale,
                             const int32_t* segment_end_offsets, const int32_t* segment_expert, int64_t M, int64_t N,
                             int64_t K, int64_t n_segments, int64_t n_experts, int32_t b_format, void* out,
                             int out_dtype, void* workspace, int64_t workspace_bytes, void* stream);
int mxgg_grouped_mm_segments_cfg(const void* a, const void* b, const void* a_scale, const void* b_scale,
                                 const int32_t* segment_end_offsets, const int32_t* segment_expert, int64_t M,
                                 int64_t N, int64_t K, int64_t n_segments, int64_t n_experts, int32_t b_format,
                                 void* out, int out_dtype, const mxgg_gemm_config* config, void* workspace,
                                 int64_t workspace_bytes, void* stream);

/*
 * Forward with the output's MX quantisation fused into the epilogue: as
 * mxgg_grouped_mm_segments (segment_expert may be null: segment s uses
 * expert s, n_experts = n_segments), and every 32-column block of output row
 * r is also written as e4m3 to q_out (M, N) bytes with its e8m0 scale at
 * q_scales[r * N / 32 + block] -- bit for bit what to_mx (mxgg_quantize_mx,
 * rows mode, row-major scales) returns for the bf16 / f16 output, which is
 * rounded first.  out may be null: only the quantised outputs are written.
 * qt_out, qt_scales (or null): the output's transpose quantised along M --
 * to_mx(out.t()), what mxgg_quantize_mx's cols mode returns, the (N, M)
 * operand layout of the next weight-gradient pass -- (N, M) e4m3 and
 * (N, M/32) e8m0; needs M % 32 == 0 and every segment starting on the 32-row
 * grid (a segment off the grid sets device status bit 256 and its blocks are
 * not written).  q_out may be null when qt_out is not.
 * Needs N % 32 == 0, 16-byte aligned q_out / qt_out, out_dtype bf16 or f16.
 * Rows past segment_end_offsets[n_segments-1] (columns, for qt_out) are not
 * written.  The workspace is
 * mxgg_grouped_mm_segments_workspace_size's.  Replaces the pair
 * triton_mxfp8_grouped_mm + to_mx of its output (kernels/forward.py:461-606,
 * utils.py:67-105) that the next layer's forward runs.
 */
int mxgg_grouped_mm_mx(const void* a, const void* b, const void* a_scale, const void* b_scale,
                       const int32_t* segment_end_offsets, const int32_t* segment_expert, int64_t M, int64_t N,
                       int64_t K, int64_t n_segments, int64_t n_experts, int32_t b_format, void* out, int out_dtype,
                       void* q_out, void* q_scales, void* qt_out, void* qt_scales, void* workspace,
                       int64_t workspace_bytes, void* stream);
int mxgg_grouped_mm_mx_cfg(const void* a, const void* b, const void* a_scale, const void* b_scale,
                           const int32_t* segment_end_offsets, const int32_t* segment_expert, int64_t M, int64_t N,
                           int64_t K, int64_t n_segments, int64_t n_experts, int32_t b_format, void* out,
                           int out_dtype, void* q_out, void* q_scales, void* qt_out, void* qt_scales,
                           const mxgg_gemm_config* config, void* workspace, int64_t workspace_bytes, void* stream);

/*
 * Expert-parallel forward with the combine fused into the epilogue: as
 * mxgg_grouped_mm_segments, but segment s's output rows are stored to
 * destination segment_dst[s] from row segment_dst_row[s] on, where
 * destination d is the (rows dst_rows[d], N) output buffer dst_out[d] --
 * typically rank d's output, mapped into this process by mxgg_ipc_open.
 * The local destination (local_dst) is written with TMA stores, the others
 * over NVLink, so the return all-to-all overlaps the math tile by tile.
 * With dst_inbox (a HOST array of n_dst buffers as large as the outputs, or
 * null), a peer's full 32-row x 64-byte blocks travel as contiguous 2 KB
 * bulk copies into its inbox, which its owner unpacks with
 * mxgg_inbox_unpack; this needs every segment to start on a 32-row boundary
 * of its destination and N * element size % 64 == 0 (otherwise, and for
 * partial blocks, rows are stored in place with 16-byte stores).  dst_out
 * and dst_rows are HOST arrays of n_dst <= 8 entries; segment_dst /
 * segment_dst_row are device int32 arrays.  Output rows must be 16-byte
 * aligned (N * element size % 16 == 0).  Peers may read their outputs (and
 * unpack their inboxes) after a later mxgg_peer_barrier on every rank.  No
 * counterpart in the reference (its path is single-GPU).
 */
int mxgg_grouped_mm_ep(const void* a, const void* b, const void* a_scale, const void* b_scale,
                       const int32_t* segment_end_offsets, const int32_t* segment_expert, const int32_t* segment_dst,
                       const int32_t* segment_dst_row, int64_t M, int64_t N, int64_t K, int64_t n_segments,
                       int64_t n_experts, int32_t b_format, void* const* dst_out, const int64_t* dst_rows,
                       void* const* dst_inbox, int32_t n_dst, int32_t local_dst, const void* a_atoms,
                       const int32_t* src_flags, int32_t src_epoch, const int32_t* segment_src,
                       const void* a_self, int64_t a_self_rows, int32_t self_src, int64_t self_row_base,
                       void* q_out, void* q_scales, int out_dtype, void* workspace, int64_t workspace_bytes,
                       void* stream);

/* Streaming dispatch for mxgg_grouped_mm_ep.  a_atoms (or null): the A
 * scales already packed into the GEMM's 128x4 atoms by the senders
 * (mxgg_pack_a_atoms, at least mxgg_ep_atom_bytes(M, K, n_segments) bytes,
 * 256-byte aligned); src_flags (or null): a device int32 array of 32 slots
 * indexed by source id; the GEMM loads a segment's rows only after
 * src_flags[source id of s] has reached src_epoch (a bounded wait, status
 * bit 128 on timeout).  Senders publish with mxgg_peer_signal after their
 * copies, so segments start as their rows land instead of after a barrier.
 * segment_src (device int32, or null when every segment's source is its
 * destination segment_dst): the source id of each segment's rows, in
 * [0, 32): the sending rank, or rank + n_dst * piece when a sender's rows
 * travel in pieces that it flags one by one.
 * a_self (or null): an (a_self_rows, K) e4m3 tensor holding the rows of
 * source self_src, read in place -- segment rows of that source at receive
 * row r are a_self row r + self_row_base -- so a rank's own rows need no copy
 * and no wait.
 * q_out, q_scales (or null): when every row stays on this GPU (dst_rows is 0
 * for every destination but local_dst), the local output is also written in
 * MXFP8 as by mxgg_grouped_mm_mx -- q_out (dst_rows[local_dst], N) e4m3,
 * q_scales (dst_rows[local_dst], N/32) e8m0 -- and dst_out[local_dst] may
 * be null (quantised rows only). */
int32_t mxgg_query_tile_m(void);
int64_t mxgg_ep_atom_bytes(int64_t M, int64_t K, int64_t n_segments);
/* Packs the scales of `rows` rows (a_scale (rows, K/32) row-major) grouped
 * in n_segments segments (device cumulative ends, relative to the first row)
 * into the blocked layout of forward A scales -- 128-row slabs, a new slab at
 * every segment start, [slab][ceil(K/128)][512 B] -- numbered from 0, at
 * `out` (typically inside a peer's atom buffer, at the slab where this
 * sender's segments start in the receiver's order: the sum of
 * ceil(rows / 128) over the receiver's earlier segments). */
int mxgg_pack_a_atoms(const void* a_scale, const int32_t* segment_end_offsets, int64_t rows, int64_t K,
                      int64_t n_segments, void* out, void* stream);
/* n_dst <= 8 such packs in one launch, as a sender makes them for all its
 * destinations: pack i takes rows [first_row[i], first_row[i] + rows[i]) of
 * a_scale ((rows, K/32) row-major), split by the n_segments[i] device
 * cumulative ends segment_end_offsets[i], and writes out[i].  HOST arrays
 * of n_dst entries; packs with rows[i] == 0 are skipped.  The same bytes as
 * n_dst calls of mxgg_pack_a_atoms, with one launch instead of n_dst. */
int mxgg_pack_a_atoms_multi(const void* a_scale, int64_t K, int32_t n_dst, const int64_t* first_row,
                            const int64_t* rows, const int32_t* const* segment_end_offsets,
                            const int64_t* n_segments, void* const* out, void* stream);
/* Writes `epoch` into `slot` (usually a peer's flag array) once everything
 * earlier on `stream` is done, as a stream memory operation
 * (cuStreamWriteValue32, with its memory barrier): no kernel, so no SM is
 * needed, and a GEMM filling the GPU while it waits for such flags from its
 * peers cannot hold it back. */
int mxgg_peer_signal(void* slot, int32_t epoch, void* stream);

/* Sums the n replicas of an array of `elems` elements of `dtype`
 * (MXGG_DTYPE_BF16 / F16 / F32) that n GPUs hold, one copy each -- the
 * weight gradients of a replicated expert -- in place over NVLink.  bufs is
 * a HOST array of the n replicas' buffers as this process addresses them
 * (its own, and the peers' mapped by mxgg_ipc_open), bufs[me] this GPU's.
 * Replica `me` takes its 1/n share of the array's 16-byte chunks: loads them
 * from every replica, adds in fp32 in replica order 0..n-1, rounds once and
 * stores the sum into every replica, so all copies end bit-identical.  Every
 * replica calls it with the same bufs order, n and elems and its own `me`,
 * between two mxgg_peer_barrier calls over the replicas (the first publishes
 * the inputs, the second the sums).  elems * element size must be a multiple
 * of 16 and the buffers 16-byte aligned; n <= 8.  The reference has no
 * multi-GPU path; this replaces an all-reduce over the replica group. */
int mxgg_replica_sum(void* const* bufs, int32_t n, int32_t me, int64_t elems, int dtype, void* stream);

/* Copies the listed 32-row blocks (device int32 row-block indices) of an
 * inbox filled by peers' mxgg_grouped_mm_ep into the row-major output whose
 * rows are row_bytes long (a multiple of 64). */
int mxgg_inbox_unpack(const void* inbox, void* out, const int32_t* row_blocks, int64_t n_row_blocks,
                      int64_t row_bytes, void* stream);

/* Device memory shared between the processes of one node (CUDA IPC).
 * mxgg_ipc_alloc: cudaMalloc + zero-fill + a 64-byte handle another process
 * can open with mxgg_ipc_open (peer access enabled on first use).  Close what
 * you opened before the owner frees it. */
int mxgg_ipc_alloc(int64_t bytes, void** ptr, void* handle);
int mxgg_ipc_free(void* ptr);
int mxgg_ipc_open(const void* handle, void** ptr);
int mxgg_ipc_close(void* ptr);

/* One cudaMemcpyAsync (peer copies travel over NVLink on a copy engine). */
int mxgg_copy_async(void* dst, const void* src, int64_t bytes, void* stream);

/* Cross-GPU barrier on `stream`: writes `epoch` into slot `rank` of every
 * rank's flag array (flags[r] = rank r's array of `world` int32, HOST array
 * of device pointers), then waits until this rank's own array holds `epoch`
 * (or later) in every slot.  Every rank calls it with the same epoch, which
 * must grow from call to call (flag arrays start at 0).  Work earlier on the
 * stream is visible to peers' work after their barrier.  The wait gives up
 * after 1 s and sets bit 64 in the device status word. */
int mxgg_peer_barrier(void* const* flags, int32_t world, int32_t rank, int32_t epoch, void* stream);

/*
 * Weight-gradient grouped GEMM: out[g] = GO_t[:, group g] @ X_t[:, group g]^T.
 * Replaces triton_mxfp8_wgrad (reference kernels/backward.py:217-305).
 *   go_t     (N, M) e4m3 (quantised along tokens)   go_scale (N, M/32)
 *   ia_t     (K, M) e4m3 (quantised along tokens)   ia_scale (K, M/32)
 *   group_end_offsets (E,) int32, device, multiples of 32 (the reference's
 *            own requirement: a 32-token scale block never spans two groups)
 *   out      (E, N, K) of out_dtype; empty groups produce zeros.
 *   workspace  >= mxgg_wgrad_workspace_size(N, K, M, E) bytes.
 * Requirements: M % 32 == 0; go_t, ia_t 16-byte aligned; 1 <= E <= 256.
 */
int mxgg_wgrad(const void* go_t, const void* go_scale, const void* ia_t, const void* ia_scale,
               const int32_t* group_end_offsets, int64_t N, int64_t K, int64_t M, int64_t E, void* out,
               int out_dtype, void* workspace, int64_t workspace_bytes, void* stream);
int mxgg_wgrad_cfg(const void* go_t, const void* go_scale, const void* ia_t, const void* ia_scale,
                   const int32_t* group_end_offsets, int64_t N, int64_t K, int64_t M, int64_t E, void* out,
                   int out_dtype, const mxgg_gemm_config* config, void* workspace, int64_t workspace_bytes,
                   void* stream);

/*
 * mxgg_wgrad, accumulating: out[g] += GO_t[:, group g] @ X_t[:, group g]^T
 * into an existing fp32 (E, N, K) gradient buffer (gradient accumulation
 * across micro-batches without a separate add pass).  Each element is added
 * once per call (TMA reduce-add), so the result is deterministic.  Workspace
 * as mxgg_wgrad.  No counterpart in the reference, which always allocates a
 * fresh output (backward.py:251).
 */
int mxgg_wgrad_accumulate(const void* go_t, const void* go_scale, const void* ia_t, const void* ia_scale,
                          const int32_t* group_end_offsets, int64_t N, int64_t K, int64_t M, int64_t E, float* out,
                          void* workspace, int64_t workspace_bytes, void* stream);
int mxgg_wgrad_accumulate_cfg(const void* go_t, const void* go_scale, const void* ia_t, const void* ia_scale,
                              const int32_t* group_end_offsets, int64_t N, int64_t K, int64_t M, int64_t E,
                              float* out, const mxgg_gemm_config* config, void* workspace, int64_t workspace_bytes,
                              void* stream);

/*
 * MX quantiser, FLOOR scaling, e4m3 elements, 32-element blocks.
 * Bit-exact with the reference's to_mx (utils.py:67-105).
 *   x        (rows, cols) of x_dtype, contiguous.
 *   mode     MXGG_QUANT_ROWS: blocks along cols (cols % 32 == 0);
 *              q (rows, cols), scales (rows, cols/32).
 *            MXGG_QUANT_COLS: blocks along rows (rows % 32 == 0), output
 *              transposed: q (cols, rows), scales (cols, rows/32) -- the
 *              reference's to_mx(x.t().contiguous()) in one pass.
 *   scale_layout MXGG_SCALE_ROW_MAJOR or MXGG_SCALE_BLOCKED (the caller
 *              zero-fills the padding of a blocked buffer).
 */
/* Quantise-on-dispatch: MXFP8 rows mode of the gathered rows
 * x[row_index[i]] (zeros where row_index[i] is negative -- padding -- or
 * not below in_rows), so the routing gather and to_mx are one pass.  q (n_rows, cols) e4m3, scales (n_rows, cols/32) row-major.
 * Bit-exact with to_mx of the gathered rows.  No counterpart in the
 * reference. */
int mxgg_quantize_mx_gather(const void* x, int x_dtype, int64_t in_rows, const int32_t* row_index, int64_t n_rows,
                            int64_t cols, void* q, void* scales, void* stream);

/* MoE combine: out[t] = sum_j weights[t*k + j] * y[pos[t*k + j]] (bf16 rows of
 * length N, fp32 sum in choice order, bf16 out); positions outside [0, y_rows)
 * contribute nothing.  pos int64, weights fp32, both (tokens, k) on the
 * device.  No counterpart in the reference. */
int mxgg_combine_topk(const void* y, int64_t y_rows, const int64_t* pos, const float* weights, int64_t tokens,
                      int64_t N, int32_t k, void* out, void* stream);

/* MXFP4 quantiser (rows mode): FLOOR scaling with emax 2, e2m1 elements
 * packed two per byte (element 2i in the low nibble) into q (rows, cols/2),
 * scales (rows, cols/32) e8m0.  Values saturate to +-6; NaN becomes +6 (e2m1
 * has no NaN).  No counterpart in the reference (its to_mx is e4m3 only). */
int mxgg_quantize_mx_fp4(const void* x, int x_dtype, int64_t rows, int64_t cols, void* q, void* scales,
                         int scale_layout, void* stream);

int mxgg_quantize_mx(const void* x, int x_dtype, int64_t rows, int64_t cols, void* q, void* scales,
                     int mode, int scale_layout, void* stream);

/* The rows mode of mxgg_quantize_mx with the scales written in the segmented
 * blocked layout (see MXGG_SCALE_BLOCKED), ready for a grouped GEMM called
 * with scale_layout MXGG_SCALE_BLOCKED: the segments are the groups
 * (segment_end_offsets, device int32 cumulative ends, n_segments <= 256) or,
 * with segment_end_offsets null, n_segments uniform segments of segment_rows
 * rows (a weight tensor's experts).  scales holds at least
 * mxgg_blocked_scale_bytes(rows, cols, n_segments) bytes; entries no row
 * fills are left as they are (zero-fill them for a bit-for-bit comparison
 * with torch's to_blocked).  No counterpart in the reference. */
int64_t mxgg_blocked_scale_bytes(int64_t rows, int64_t contraction, int64_t n_segments);
int mxgg_quantize_mx_blocked(const void* x, int x_dtype, int64_t rows, int64_t cols, void* q, void* scales,
                             const int32_t* segment_end_offsets, int64_t n_segments, int64_t segment_rows,
                             void* stream);

/*
 * Routing tables of the reference's _build_expt_data (forward.py:340-365),
 * built on the device: out must hold 2*E + 1 + cdiv(M, block_m) + max(E-1, 0)
 * int32: [hist (E) | start offsets (E) | total tiles (1) | tile map], tile
 * map entries (block << 16) | group, or -1 past the last tile.
 */
int mxgg_build_tile_map(const int32_t* group_end_offsets, int64_t E, int64_t M, int32_t block_m, int32_t* out,
                        void* stream);

/* Process default tile configuration (0 = automatic): tile_m in {128 (one
 * CTA per tile), 256 (a CTA pair per tile)}, tile_n in {128, 256},
 * group_m >= 1 rasterisation band in m-tiles.  Every call takes a snapshot
 * of the defaults under a lock; a call's own mxgg_gemm_config overrides
 * them, which is how concurrent callers choose different configs. */
int mxgg_set_tile_config(int32_t tile_m, int32_t tile_n, int32_t group_m);

/* Process default work schedule (a call's mxgg_gemm_config overrides it).  Output tiles are
 * dealt to the persistent CTA pairs in rounds.  TILES (what DEFAULT means)
 * deals every tile whole.  With SPLIT_TAIL the tiles of the last, partial
 * round are cut along the contraction into pieces for the pairs that would
 * otherwise idle, and the last piece to finish sums the fp32 partials in a
 * fixed order (results do not depend on timing); that schedule runs a
 * kernel build with the split machinery compiled in, which measured ~3 %
 * slower per stage, so it pays only where the tail round is long.
 * split_max caps the pieces per tile (0: about the square root of the
 * tile's 128-element stages; else 2..64).  No counterpart in the reference. */
enum { MXGG_SCHED_DEFAULT = 0, MXGG_SCHED_TILES = 1, MXGG_SCHED_SPLIT_TAIL = 2 };
int mxgg_set_schedule(int32_t schedule, int32_t split_max);

/* Limit of every bounded device-side wait (pipeline barriers, peers' rows in
 * mxgg_grouped_mm_ep, mxgg_peer_barrier), in ns of %globaltimer: 1 ms .. 60 s,
 * 0 restores the default 1 s.  A wait that runs out sets its bit in the
 * device status word and the kernel returns; the call's output is then
 * incomplete.  Process-wide; each call reads it when it is enqueued.  No
 * counterpart in the reference (its kernels have no device-side waits). */
int mxgg_set_wait_limit(int64_t ns);
int64_t mxgg_wait_limit(void);

/* Error bits raised by device-side bounded waits since the last clear
 * (0 = none; bit 256: a transposed quantised output met a group off the
 * 32-row grid).  Synchronises `stream`.  clear != 0 resets the word. */
int mxgg_device_status(uint32_t* status_out, int clear, void* stream);

const char* mxgg_last_error(void);
int32_t mxgg_version(void);
/* Digest of the sources this library was built from (build.py embeds it);
 * the Python loader refuses a library whose digest differs from the sources
 * beside it. */
const char* mxgg_build_id(void);

#ifdef __cplusplus
}
#endif

#endif /* MXGG_H_ */
