/*
 * li_b200.h — C ABI of the B200-native (sm_100a) AR-aware 3D block-sparse
 * attention backend.
 *
 * Every entry point takes plain device pointers, element strides, sizes and a
 * CUDA stream (passed as `void*`, i.e. a cudaStream_t / CUstream; NULL is the
 * legacy default stream). Calls are asynchronous on that stream, allocate no
 * memory (except the setup-time li_ipc_alloc), and never synchronise the host.
 * Each returns an li_status; on a non-zero status nothing was launched and
 * li_last_error() describes why.
 *
 * Tensor views (li_view4 / li_view5) describe strided tensors. Strides are in
 * elements. The innermost dimension (head dim D) must be contiguous.
 *
 * Layout vocabulary (names follow the reference):
 *   raster  [B, H, L, D] with L = T*LH*LW tokens in (t, h, w) order;
 *   tiled   [B, H, Nblk, bs, D]: 3D blocks of bs = tt*th*tw tokens, blocks in
 *           (nt, nh, nw) order, tokens inside a block in (tt, th, tw) order,
 *           partial blocks zero-filled.
 * Reference paths below are relative to the reference project root.
 */
#ifndef LI_B200_H
#define LI_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
typedef int32_t li_status;
#define LI_OK                 0
#define LI_ERR_INVALID_ARG    1  /* null pointer, bad enum, bad parameter      */
#define LI_ERR_SHAPE          2  /* inconsistent or unsupported shape          */
#define LI_ERR_STRIDE         3  /* D not contiguous / stride not encodable    */
#define LI_ERR_ALIGNMENT      4  /* pointer or stride not 16-byte aligned      */
#define LI_ERR_OUT_OF_BOUNDS  5  /* an index outside its range                 */
#define LI_ERR_UNSUPPORTED    6  /* dtype / head dim / block size not built    */
#define LI_ERR_CUDA           7  /* a CUDA runtime or driver call failed       */
#define LI_ERR_TIMEOUT        8  /* a bounded device-side wait gave up         */

/* Bits OR-ed into the optional device error word (`err_word`) by kernels. */
#define LI_DEVERR_BAD_INDEX   1u  /* a block index outside [0, n_kv_blocks)    */
#define LI_DEVERR_TIMEOUT     2u  /* an mbarrier wait exceeded its bound       */
#define LI_DEVERR_RANGE       4u  /* an fp32 attention operand beyond the fp16
                                     range of the fp32 path (set by the Python
                                     layer's operand conversion)               */

/* ---- enums ------------------------------------------------------------- */
#define LI_DTYPE_BF16 0
#define LI_DTYPE_FP16 1
#define LI_DTYPE_FP32 2

#define LI_METRIC_COSINE      0  /* 'cosine'                                  */
#define LI_METRIC_SCALED_DOT  1  /* 'scaled_dot_product'                      */
#define LI_METRIC_DOT         2  /* any other string (plain dot product)      */

#define LI_SELECT_DECODE 0  /* fast_generate_indices: protect recent blocks    */
#define LI_SELECT_BIDIR  1  /* generate_prefill_indices: protect neighbours    */

/* ---- tensor views ------------------------------------------------------ */
typedef struct li_view4 {
  void*   data;
  int64_t shape[4];
  int64_t stride[4];   /* elements */
  int32_t dtype;       /* LI_DTYPE_* */
} li_view4;

typedef struct li_view5 {
  void*   data;
  int64_t shape[5];
  int64_t stride[5];   /* elements */
  int32_t dtype;
} li_view5;

typedef struct li_index_view {      /* int32 [B, H, Nq_blk, S] + counts [B, H, Nq_blk] */
  int32_t* indices;
  int64_t  shape[4];
  int64_t  stride[4];
  int32_t* counts;
  int64_t  count_stride[3];
} li_index_view;

/* 3D block geometry of a raster tensor. */
typedef struct li_grid3d {
  int32_t T, LH, LW;   /* frames, latent height, latent width              */
  int32_t tt, th, tw;  /* tile (block) shape                               */
} li_grid3d;

/* ---- library ----------------------------------------------------------- */
const char* li_version(void);
/* Message of the last failed call on this host thread ("" if none). */
const char* li_last_error(void);
/* Kernels this process has launched through the library so far (all devices,
 * all threads). A diagnostic with no reference counterpart: benchmarks read it
 * before and after a timed region. */
uint64_t li_kernel_launches(void);

/* ---- (a1, a2, a3, a10) tiling + pooling + frame gather ------------------
 * Replaces launch_q_prep / _fused_q_prep_kernel
 *   (hy-worldplay/files/hyvideo/models/transformers/modules/ar_sparse_operation.py:26-70,166-181)
 * and launch_kv_prep / _fused_kv_prep_kernel (same file :75-122,183-202; copies in
 *   bi_sparse_operation_for_KV_cache.py:27-126,168-200 and
 *   matrix-game-3.0/files/wan/modules/bi_sparse_operation.py:25-107,142-166).
 *
 * Tiles one or two raster streams (src0, optional src1 — K and V) into the
 * tiled layout at block offset `dst_block_offset` (the text blocks precede the
 * visual ones), and writes the per-block mean of src0 (fp64-accumulated, then
 * fp32 / bs, rounded to the dtype) at block offset `pool_block_offset`.
 * `frame_ids` (optional, int32 device array of length grid.T) maps logical frame
 * t to the physical frame of src0/src1 it is read from — the memory-pruning
 * gather (a10) fused into the copy; NULL means identity. Either of dst0 or pool
 * may be NULL (pool only / tile only). dst1 must be given iff src1 is.
 */
li_status li_tile_pool(const li_view4* src0, const li_view4* src1, const int32_t* frame_ids,
                       li_grid3d grid, li_view5* dst0, li_view5* dst1,
                       int64_t dst_block_offset, li_view4* pool, int64_t pool_block_offset,
                       void* stream);

/* Pool-only form of li_tile_pool for one stream, optionally normalised: with
 * `normalized` != 0 the stored row is F.normalize(mean, dim=-1) with the
 * selection's rounding chain (sqrt of the fp64 sum of squares -> fp32 -> dtype,
 * clamped at dtype(1e-12), fp32 quotient -> dtype), i.e. li_normalize_rows of
 * the li_tile_pool mean, bit for bit, in one launch — the block mean of
 * launch_q_prep / launch_kv_prep plus the F.normalize of the 'cosine' metric
 * (ar_sparse_operation.py:252, bi_sparse_operation.py:197). */
li_status li_pool_blocks(const li_view4* src, const int32_t* frame_ids, li_grid3d grid, li_view4* pool,
                         int64_t pool_block_offset, int32_t normalized, void* stream);

/* Several li_pool_blocks jobs in one launch (1 to 4 jobs sharing the dtype and
 * head dim; each keeps its own source, grid, pool and normalisation) — e.g. the
 * q pool and the changed key-pool rows of one attention call, which the
 * reference computes in its q-prep and kv-prep launches
 * (ar_sparse_operation.py:166-202). Results are those of one li_pool_blocks
 * call per job, bit for bit. */
typedef struct li_pool_job {
  const li_view4* src;
  const int32_t* frame_ids;       /* optional, as in li_pool_blocks            */
  li_grid3d grid;
  li_view4* pool;
  int64_t pool_block_offset;
  int32_t normalized;
} li_pool_job;
li_status li_pool_blocks_multi(const li_pool_job* jobs, int32_t n_jobs, void* stream);

/* Text K/V into the first blocks of the tiled K/V buffers, zero-padded to a
 * block multiple — replaces the F.pad + copy_ at ar_sparse_operation.py:337-344
 * (bi_sparse_operation_for_KV_cache.py:369-375; bi_sparse_operation.py:279-286).
 * src0/src1: [B, H, N_txt, D]; writes ceil(N_txt/bs) blocks at block 0. */
li_status li_text_blocks(const li_view4* src0, const li_view4* src1, int32_t bs,
                         li_view5* dst0, li_view5* dst1, void* stream);

/* (a8) Untile: tiled [B,H,Nblk,bs,D] -> raster [B,H,T*LH*LW,D], padded rows
 * dropped — replaces launch_untile / _fused_untile_kernel
 * (ar_sparse_operation.py:127-161,204-218; bi_sparse_operation.py:109-140,168-177). */
li_status li_untile(const li_view5* src, li_grid3d grid, li_view4* dst, void* stream);

/* (a10) Memory-pruning gather on its own: dst[:, :, f] = src[:, :, frame_ids[f]]
 * for frames of `frame_tokens` tokens — the retained-frame selection of
 * hy-worldplay/patches/0001-integrate-acceleration.patch:3213-3221
 * (`latents[:, :, selected_frame_indices]`) and
 * matrix-game-3.0/patches/0001-integrate-acceleration.patch:447-457, applied
 * to a K/V pool. Frame ids outside [0, src_frames) are rejected on the device
 * (LI_DEVERR_BAD_INDEX in err_word; the frame is zero-filled). */
li_status li_gather_frames(const li_view4* src, const int32_t* frame_ids, int32_t n_frames,
                           int32_t frame_tokens, li_view4* dst, uint32_t* err_word,
                           void* stream);

/* ---- (a4, a5) block selection ------------------------------------------ */
typedef struct li_select_params {
  int32_t mode;            /* LI_SELECT_DECODE or LI_SELECT_BIDIR                   */
  int32_t metric;          /* LI_METRIC_*                                           */
  int32_t tt, th, tw;      /* params['tile_size']                                   */
  int32_t grid_q[3];       /* (nt_q, nh, nw) — decode uses grid_q[1..2] for n_prot  */
  int32_t grid_k[3];       /* (nt_k, nh, nw) — bidir neighbour geometry             */
  int32_t text_len;        /* text tokens; ceil(text_len/bs) blocks are prepended   */
  int32_t recent_protect;  /* decode: frames protected at the end of the key grid   */
  double  topk_ratio;      /* params['topk_ratio']                                  */
  int32_t min_budget;      /* bidir: lower bound of the budget (reference: 7)       */
  int32_t q_block_offset;  /* bidir: key-grid position of query row 0 (0 = square)  */
} li_select_params;

/* Budget (number of visual blocks kept per query row) the selection will use,
 * so the caller can size the index tensor: ntxt + budget columns. */
li_status li_select_budget(const li_select_params* p, int64_t n_q_blocks, int64_t n_k_blocks,
                           int32_t* n_text_blocks, int32_t* budget);

/* Replaces fast_generate_indices (ar_sparse_operation.py:223-284) and
 * generate_prefill_indices (bi_sparse_operation_for_KV_cache.py:220-296,
 * bi_sparse_operation.py:179-234) on pooled inputs [B, H, N, D].
 * Writes indices [B,H,Nq,ntxt+budget] (int32, ascending, text blocks first) and
 * counts [B,H,Nq]. `score_bias` (optional fp32 [B,H,Nq,Nk] view, harness
 * extension) is added to the similarity before the protection bias.
 * `rank_out` (optional fp32 [B,H,Nq,Nk]) receives the ranking scores.
 * `workspace` (optional, li_select_workspace_bytes() bytes, 16-byte aligned)
 * lets the scores and the top-k run as two wide kernels; without it one
 * kernel does both (same results, bit for bit). */
li_status li_select_blocks(const li_view4* q_pool, const li_view4* k_pool,
                           const li_select_params* p, const li_view4* score_bias,
                           li_index_view* out, li_view4* rank_out,
                           void* workspace, int64_t workspace_bytes, void* stream);

/* Bytes of the optional selection workspace (0 when the shape cannot use it). */
li_status li_select_workspace_bytes(int64_t batch, int64_t heads, int64_t n_q_blocks, int64_t n_k_blocks,
                                    int64_t* bytes);

/* Size of the scratch array behind li_select_blocks_static. */
#define LI_SELECT_STATIC_SCRATCH_BYTES (8ll << 20)

/* li_select_blocks' two-kernel path with its scratch in a fixed array of the
 * library's own global memory (LI_SELECT_STATIC_SCRATCH_BYTES), so the call
 * allocates nothing: for hosts with no device allocator to hand a workspace
 * from. No reference counterpart — the reference always allocates its score
 * tensors through torch.
 * - Same arguments and results (bit for bit) as li_select_blocks with a
 *   workspace; nothing in the scratch has to start at zero.
 * - Shapes needing more than batch*heads*n_q_blocks*n_k_blocks*4 =
 *   LI_SELECT_STATIC_SCRATCH_BYTES bytes return LI_ERR_UNSUPPORTED.
 * - The first call on each device looks the array up (and may load the
 *   library's module); make it, with that device current, before any stream
 *   capture.
 * - One array per device: calls that may run at the same time on one device
 *   (different streams, or host threads without ordering) race on it. */
li_status li_select_blocks_static(const li_view4* q_pool, const li_view4* k_pool,
                                  const li_select_params* p, const li_view4* score_bias,
                                  li_index_view* out, li_view4* rank_out, void* stream);

/* Row-wise F.normalize (dim=-1) of pooled rows, with the selection kernel's
 * exact rounding chain: y = dtype(x / max(dtype(sqrt(fp32(sum x^2))), dtype(1e-12))).
 * Cosine selection equals the plain-dot selection of normalised pools, so the
 * pipeline normalises each pool once here instead of in every selection CTA —
 * the F.normalize calls of ar_sparse_operation.py:252 / bi_sparse_operation.py:197. */
li_status li_normalize_rows(const li_view4* x, li_view4* y, void* stream);

/* The ranking step alone on given ranking scores (fp32 [B,H,Nq,Nk] holding
 * `dtype` values): top-`k` by the dtype's radix order, ties to the lowest
 * index, sorted ascending, offset by ntxt = ceil(text_len/bs) with 0..ntxt-1
 * prepended — torch.topk + torch.sort + cat at ar_sparse_operation.py:274-282. */
li_status li_rank_blocks(const li_view4* rank_scores, int32_t score_dtype, int32_t k,
                         int32_t text_len, int32_t bs, li_index_view* out, void* stream);

/* ---- (a6, a7, a8) block-sparse attention forward ----------------------- */
/* Split-KV workspace. The attention runs one CTA per query block per SM; when
 * the last wave of a launch would hold only a few blocks, the lists of those
 * blocks are split over several CTAs that write fp32 partials (O, row max,
 * row sum) to a caller-provided device workspace, merged by a second kernel.
 * This returns the bytes the attention entry points will use for that shape
 * (0 = no split; never more than one wave of partials). A smaller or NULL
 * workspace is allowed and simply disables the split. No reference
 * counterpart (the reference always launches one program per 128 query rows). */
li_status li_sparse_attn_workspace_bytes(int64_t batch, int64_t heads, int64_t n_q_blocks,
                                         int64_t max_blocks_per_row, int32_t head_dim, int32_t block_size,
                                         int64_t* bytes);

/* Tiled form — replaces longcat_flash_attn / _attn_fwd_bsa_align
 * (hy-worldplay/.../longcat_kernel.py:27-233; matrix-game-3.0/.../longcat_kernel.py:28-190).
 * q [B,H,Q_len,D], k/v [B,H,K_len,D] in the tiled order, K_len % bs == 0.
 * Query block i (rows i*bs .. i*bs+bs-1) attends to key blocks
 * indices[b,h,i,0:counts[b,h,i]]. o has q's shape; lse (optional fp32
 * [B,H,Q_len], log2 domain like the reference's M buffer) may be NULL.
 * D in {64, 128}; bs in {32, 64, 128, 256} (the reference takes any power of two;
 * a 256-token block runs as two 128-row halves, a block of 64 or 32 query rows
 * fills the 128-row MMA tile with zero rows); q/k/v/o bf16 or fp16 (all the
 * same). */
li_status li_sparse_attn_tiled(const li_view4* q, const li_view4* k, const li_view4* v,
                               const li_index_view* idx, int32_t bs, float sm_scale,
                               li_view4* o, float* lse, uint32_t* err_word,
                               void* workspace, int64_t workspace_bytes, void* stream);

/* Raster form (fused tile -> attention -> untile): reads q and the visual K/V
 * straight from their raster layouts in 3D blocks (zero-filled past the grid
 * edges, as the tiled path pads), the text K/V (optional, [B,H,N_txt,D]) as
 * ceil(N_txt/bs) leading blocks, and writes o in q's raster layout, dropping
 * padded rows. Key block j < ntxt is text block j; j >= ntxt is visual block
 * j - ntxt of grid_k. Same math as tiling + li_sparse_attn_tiled + untiling. */
li_status li_sparse_attn_raster(const li_view4* q, li_grid3d grid_q,
                                const li_view4* k_txt, const li_view4* v_txt,
                                const li_view4* k_vis, const li_view4* v_vis, li_grid3d grid_k,
                                const li_index_view* idx, float sm_scale,
                                li_view4* o, float* lse, uint32_t* err_word,
                                void* workspace, int64_t workspace_bytes, void* stream);

/* ---- (e) head-sharded stack: all-to-all over NVLink peer memory ----------
 * No reference counterpart inside the sparse op; replaces the NCCL exchange of
 * the upstream Ulysses re-layout (all_to_all_4D, hy patch:646-654,744-745)
 * around it. Buffers are plain CUDA IPC allocations (no multicast object). */
#define LI_A2A_MAX_RANKS    8
#define LI_IPC_HANDLE_BYTES 64

/* Setup-time only (not per call): a zeroed device allocation of `bytes` and
 * its IPC handle (LI_IPC_HANDLE_BYTES bytes written to handle_out). */
li_status li_ipc_alloc(int64_t bytes, void** ptr, void* handle_out);
/* Maps a peer process's allocation from its IPC handle (peer access enabled). */
li_status li_ipc_open(const void* handle, void** ptr);
li_status li_ipc_close(void* ptr);
li_status li_ipc_free(void* ptr);

typedef struct li_a2a_desc {
  const void* src;                      /* local send buffer                          */
  int64_t src_chunk_stride;             /* bytes between the chunks for rank p        */
  int64_t src_row_stride;               /* bytes between rows of a chunk              */
  int64_t rows, row_bytes;              /* rows per chunk, bytes per row (x16)        */
  void* dst[LI_A2A_MAX_RANKS];          /* receive buffer of every rank (IPC-mapped)  */
  int64_t dst_bytes;                    /* size of each receive buffer                */
  int64_t dst_offset;                   /* where this rank's chunk lands, bytes       */
  int64_t dst_row_stride;               /* bytes between its rows there               */
  uint32_t* flags[LI_A2A_MAX_RANKS];    /* flag array of every rank (world u32 each)  */
  uint32_t* my_flags;                   /* this rank's flag array (= flags[rank])     */
  uint32_t* counter;                    /* this rank's zeroed u32 ticket counter      */
  uint32_t* err_word;                   /* optional device error word                 */
  uint32_t* epoch_word;                 /* optional: the epoch kept on the device     */
  uint32_t epoch;                       /* 1, 2, ... per call, the same on all ranks  */
  int32_t world, rank;
  /* Optional split rows (0: none). With split_bytes > 0 the first split_bytes
   * of every row go to dst as above and the remaining row_bytes - split_bytes
   * to dst2[p] + dst2_offset + r * dst2_row_stride (all 16-byte multiples). */
  int64_t split_bytes;
  void* dst2[LI_A2A_MAX_RANKS];         /* second destination of every rank          */
  int64_t dst2_bytes;                   /* size of each second destination            */
  int64_t dst2_offset, dst2_row_stride; /* bytes                                      */
} li_a2a_desc;

/* Chunk p of `src` (rows x row_bytes) -> rank p's receive buffer at dst_offset,
 * rows dst_row_stride apart, with 16-byte peer stores; returns (on the stream)
 * once every rank's chunk for this rank has landed. Every rank must make the
 * same sequence of calls; one descriptor's counter serves one stream. A peer
 * that does not join within 2 s sets LI_DEVERR_TIMEOUT and the kernel returns.
 * After LI_DEVERR_TIMEOUT the exchange's buffers must not be used again: a
 * late peer may still be writing into them while the epoch has moved on, so
 * the caller frees them and builds a new exchange (new buffers, new flags).
 * With `epoch_word` set (a zeroed u32 on this rank's device) the call's epoch is
 * *epoch_word + 1, read and stored back by the kernel, and `epoch` is ignored:
 * the launch then carries no per-call value, so a captured CUDA graph can replay
 * it. */
li_status li_a2a_push(const li_a2a_desc* desc, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* LI_B200_H */
