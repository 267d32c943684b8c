/*
 * veda_b200.h - C ABI of the B200 (sm_100a) Veda sparse-attention hot path.
 *
 * Plain pointers, sizes and a CUDA stream; no torch types. Every entry point
 * returns VEDA_OK (0) or an error code and never synchronises the device.
 * Device pointers must be on the calling thread's current CUDA device.
 * Errors found on the device (an out-of-range tile id in an index list, a
 * bounded wait that gave up) are OR-ed into a caller-owned int32 status word
 * in device memory (VEDA_STATUS_*), which the caller reads when it chooses.
 *
 * Reference interfaces replaced (veda-sparse/Veda-on-ComfyUI 0.3.1, paths
 * relative to its repository root) are cited on each declaration.
 */
#ifndef VEDA_B200_H_
#define VEDA_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VEDA_ABI_VERSION 4

/* Return codes. */
#define VEDA_OK 0
#define VEDA_ERR_INVALID 1     /* an argument is out of range or misaligned */
#define VEDA_ERR_CUDA 2        /* a CUDA runtime / driver call failed */
#define VEDA_ERR_UNSUPPORTED 3 /* the current device is not sm_100 */

/* Bits of the device status word. */
#define VEDA_STATUS_TIMEOUT 1     /* a bounded wait inside a kernel gave up */
#define VEDA_STATUS_BAD_INDEX 2   /* a tile id outside [0, n_tiles) was read */
#define VEDA_STATUS_OVERFLOW 4    /* a row kept more tiles than `width` */
#define VEDA_STATUS_BAD_COUNT 8   /* a count outside [0, width] was read */
#define VEDA_STATUS_MISALIGNED 16 /* shared memory was not 1024-byte aligned */

/* Element types. */
#define VEDA_BF16 0
#define VEDA_F16 1
#define VEDA_F32 2
#define VEDA_FP8_E4M3 3 /* predictor projections only, with per-head scales */

/* Version of this ABI (VEDA_ABI_VERSION). */
int veda_abi_version(void);

/* Message of the last error returned on the calling thread. */
const char* veda_last_error(void);

/* 1 if `device` is an sm_100 GPU this library was built for, else 0. */
int veda_device_supported(int device);

/*
 * Per-block INT8 quantisation of one tensor.
 * Replaces kernels/sage/sparse_int8.py:57-73 (_quantize_kernel) and
 * :118-133 (quantize).
 *   x        [n_slots, heads, dim] 16-bit (dtype), rows `stride_n` and heads
 *            `stride_h` elements apart, dim contiguous; dim == 128;
 *            n_slots a multiple of 128.
 *   block    64 or 128 rows per scale.
 *   out      [heads][n_slots][dim] int8 (head-major).
 *   scale    [heads][n_slots / block] fp32.
 * x * pre_scale is quantised as trunc(x / s + 0.5 sign) with s = max|x|/127
 * per (block, head), s = 1 for an all-zero block; all fp32, IEEE division.
 */
int veda_quantize(const void* x, int dtype, int64_t stride_n, int64_t stride_h,
                  int n_slots, int heads, int dim, int block, float pre_scale,
                  int8_t* out, float* scale, void* stream);

/*
 * Fused pass over Q and K: INT8 quantisation of Q (128 rows per scale,
 * `q_pre_scale` folded in) and K (64 rows per scale), and optionally the
 * TripPool features of every video tile of both.
 * Replaces sparse_int8.py:336-340 (the two quantize calls of attend) and
 * core/predictor.py:20-60 (pool_video_tiles).
 *   q, k         [n_slots, heads, 128] 16-bit, same strides.
 *   valid_count  [n_slots / 128] int32 real rows per tile (a prefix).
 *   q_i8, k_i8   [heads][n_slots][128] int8.
 *   q_scale      [heads][n_slots / 128]; k_scale [heads][n_slots / 64].
 *   feats_q/k    [heads][n_video_tiles][384] fp32 ([mean | max | min] over
 *                the real rows, 0 for empty tiles), or NULL to skip pooling.
 */
int veda_quant_pool(const void* q, const void* k, int dtype, int64_t stride_n,
                    int64_t stride_h, int n_slots, int heads,
                    const int32_t* valid_count, int n_video_tiles,
                    float q_pre_scale, int8_t* q_i8, float* q_scale,
                    int8_t* k_i8, float* k_scale, float* feats_q,
                    float* feats_k, void* stream);

/*
 * Predictor tile logits: x_hat = F @ P[h] + F[:, :128] for q and k, then
 * logits = q_hat k_hat^T / sqrt(128), fp32.
 * Replaces core/predictor.py:63-80 (tile_logits).
 *   feats_q      [heads][n_q][384] fp32; feats_k [heads][n_k][384] fp32.
 *   proj_q/k     [heads][384][128] (proj_dtype: VEDA_BF16/F16/F32).
 *   workspace    fp32 scratch of (n_q + n_k) * heads * 128 elements.
 *   Features, projections and workspace start 16-byte aligned
 *   (VEDA_ERR_INVALID otherwise).
 *   logits       [heads][n_q][n_k] fp32.
 */
int veda_tile_logits(const float* feats_q, const float* feats_k,
                     const void* proj_q, const void* proj_k, int proj_dtype,
                     int heads, int n_q, int n_k, float* workspace,
                     float* logits, void* stream);

/*
 * veda_tile_logits for projections stored in fp8 (e4m3) with one fp32 scale
 * per head, as fp8 predictor bundles keep them.
 * Replaces core/bundle.py:176-180 (dequantisation at load) and
 * core/predictor.py:63-80: each weight is used as bf16(w * scale[h]), the
 * value the reference's loader stores, so the logits equal those of
 * veda_tile_logits on the dequantised bf16 weights. The fp8 tensors cross
 * PCIe and HBM at half the bytes of bf16.
 *   proj_dtype   VEDA_FP8_E4M3 (scale_q / scale_k [heads] fp32 required) or
 *                any type of veda_tile_logits (scales ignored, may be NULL).
 * Other arguments as veda_tile_logits.
 */
int veda_tile_logits_scaled(const float* feats_q, const float* feats_k,
                            const void* proj_q, const void* proj_k,
                            int proj_dtype, const float* scale_q,
                            const float* scale_k, int heads, int n_q,
                            int n_k, float* workspace, float* logits,
                            void* stream);

/* Row limit of veda_tile_logits_static: (n_q + n_k) * heads. */
#define VEDA_STATIC_LOGITS_ROWS 16384

/*
 * veda_tile_logits that allocates nothing: its scratch (the projected
 * features) is a fixed 8 MiB device array inside this library, one per
 * device, instead of a caller workspace. This entry point has no
 * counterpart in the reference, whose predictor allocates through torch.
 *   Limit: n_q, n_k and (n_q + n_k) * heads each <= VEDA_STATIC_LOGITS_ROWS;
 *   larger calls return VEDA_ERR_INVALID before any device work (the
 *   sizes are checked before the device).
 *   Calls that overlap in time on one device (other streams or threads)
 *   share the array and race: serialise them.
 *   Each call looks up the array's address in the current device's context
 *   (so a device reset, which reloads the module, is followed correctly).
 *   The first call on a device loads the module if it is not yet loaded:
 *   make it before any stream capture.
 * Arguments and results are those of veda_tile_logits.
 */
int veda_tile_logits_static(const float* feats_q, const float* feats_k,
                            const void* proj_q, const void* proj_k,
                            int proj_dtype, int heads, int n_q, int n_k,
                            float* logits, void* stream);

/* One sparse column block of the video quadrant
 * (core/selection.py:109-128 ColumnBlock / column_blocks). */
typedef struct veda_column_block {
  int32_t start;      /* first key tile of the block */
  int32_t stop;       /* one past the last key tile */
  int32_t keeps_all;  /* 1: keep every non-empty tile of the block */
  int32_t k_lo;       /* tiles kept per row before the Bresenham extra */
} veda_column_block;

/*
 * Top-k key-tile selection straight into ascending index lists.
 * Replaces core/selection.py:132-180 (select), :184-203 (block_mask) and
 * :206-227 (tile_index_list) as the triton backend chains them
 * (backends/triton_int8.py:51), without the host synchronisation.
 *   scores     [heads][n_video][n_video] fp32, rows `score_stride_h` /
 *              `score_stride_r` elements apart.
 *   kv_ok      [n_tiles] uint8, 1 if the tile has a real row.
 *   blocks     n_blocks (1 or 2) host structs in column order.
 *   extra      [n_blocks][n_video] uint8 device array: 1 where the row keeps
 *              k_lo + 1 tiles of that block (the Bresenham pattern).
 *   index      [heads][n_tiles][width] int32, ascending, -1 past the count.
 *   count      [heads][n_tiles] int32.
 * Within a block, a row keeps its own tile (+inf), never an empty tile,
 * and otherwise the k_lo + extra highest scores; equal scores are taken in
 * ascending tile order. Global rows (>= n_video) and global columns keep
 * every non-empty tile.
 */
int veda_select(const float* scores, int64_t score_stride_h,
                int64_t score_stride_r, int heads, int n_video, int n_tiles,
                const uint8_t* kv_ok, int n_blocks,
                const veda_column_block* blocks, const uint8_t* extra,
                int width, int32_t* index, int32_t* count, int32_t* status,
                void* stream);

/*
 * Ascending index lists of a dense block mask (mask & kv_ok).
 * Replaces core/selection.py:206-227 (tile_index_list) with a fixed
 * `width` instead of the host-synchronising `count.max().item()`.
 *   mask   [heads][n_tiles][n_tiles] uint8 (torch.bool storage).
 */
int veda_mask_to_index(const uint8_t* mask, const uint8_t* kv_ok, int heads,
                       int n_tiles, int width, int32_t* index, int32_t* count,
                       int32_t* status, void* stream);

/*
 * Block-sparse INT8 attention on tcgen05 tensor cores: for every (head,
 * query tile) walks the listed key tiles, S = Qi8 Ki8^T (int32 in TMEM)
 * scaled by q_scale * k_scale (already in log2 units), online softmax with
 * exp2, O += P V in fp32 (P rounded to V's 16-bit type), out = O / l.
 * Replaces kernels/sage/sparse_int8.py:136-188 (_attention_kernel) and
 * :312-362 (attend) after quantisation.
 *   q_i8, k_i8   [heads][n_tiles * 128][128] int8 (veda_quantize layout).
 *   q_scale      [heads][n_tiles]; k_scale [heads][2 * n_tiles].
 *   v            [n_tiles * 128, heads, 128] 16-bit (v_dtype), row / head
 *                strides in elements, dim contiguous, 16-byte aligned.
 *   index/count  as veda_select; valid_count [n_tiles] int32.
 *   out          [n_tiles * 128, heads, 128] of v_dtype (strides in
 *                elements); rows of query tiles with count 0 are zero.
 */
int veda_sparse_attention(const int8_t* q_i8, const float* q_scale,
                          const int8_t* k_i8, const float* k_scale,
                          const void* v, int v_dtype, int64_t v_stride_n,
                          int64_t v_stride_h, const int32_t* index, int width,
                          const int32_t* count, const int32_t* valid_count,
                          int heads, int n_tiles, void* out,
                          int64_t out_stride_n, int64_t out_stride_h,
                          int32_t* status, void* stream);

/*
 * veda_sparse_attention for head-sharded runs: every output row is written
 * to `out` and then, while later rows are still being computed, once
 * through `out_multicast`, the NVSwitch multicast address of `out` (the
 * same byte offsets), so each GPU bound to the multicast object ends up
 * holding every rank's heads. This replaces the all-gather of the output
 * that head sharding needs (no counterpart in the reference, which runs on
 * one GPU). The caller orders the stores before reading other ranks' heads
 * with a collective on the same stream (the kernel ends with a
 * system-scope fence). `out` is this rank's view of the multicast-bound
 * buffer.
 */
int veda_sparse_attention_multicast(
    const int8_t* q_i8, const float* q_scale, const int8_t* k_i8,
    const float* k_scale, const void* v, int v_dtype, int64_t v_stride_n,
    int64_t v_stride_h, const int32_t* index, int width, const int32_t* count,
    const int32_t* valid_count, int heads, int n_tiles, void* out,
    void* out_multicast, int64_t out_stride_n, int64_t out_stride_h,
    int32_t* status, void* stream);

/*
 * veda_quant_pool on packed rows: q and k are [seq_len, heads, 128] in
 * sequence order and slot i of the tile order reads row perm[i] (< 0:
 * padding, zeros), so the gather of core/tiling.py:227-242 (gather_tiles)
 * happens in the same read. Outputs as veda_quant_pool, same bits as
 * veda_gather_tiles followed by veda_quant_pool. perm has n_slots entries.
 * The caller guarantees that q and k hold seq_len rows at the given
 * strides and that every perm entry is below seq_len: rows at or past
 * seq_len are treated as padding, but seq_len itself is not checked
 * against the tensors (raw pointers carry no extent).
 *   v, v_tiled   optional (both NULL or neither): packed V [seq_len, *,
 *                128] of q's dtype at v_stride_n / v_stride_h, copied
 *                through the same permutation and head ids into v_tiled
 *                [n_slots, heads, 128] (tile order, contiguous), the V
 *                operand of veda_sparse_attention_packed. Same bits as
 *                veda_gather_tiles of V, in the same launch as Q and K.
 *   head_ids     [heads] int32, or NULL for heads 0 .. heads - 1: output
 *                head h is input head head_ids[h], so one head group of a
 *                layer (core/plans.py:25-29 HeadGroup; core/engine.py:
 *                282-297) is quantised without a copy of q[:, group]. The
 *                caller guarantees every id is a head of q, k and v.
 */
int veda_quant_pool_packed(
    const void* q, const void* k, int dtype, int64_t stride_n,
    int64_t stride_h, int64_t seq_len, const int64_t* perm, int n_slots,
    int heads, const int32_t* valid_count, int n_video_tiles,
    float q_pre_scale, int8_t* q_i8, float* q_scale, int8_t* k_i8,
    float* k_scale, float* feats_q, float* feats_k, const void* v,
    int64_t v_stride_n, int64_t v_stride_h, void* v_tiled,
    const int32_t* head_ids, void* stream);

/*
 * veda_sparse_attention with a packed output: row `slot` of the result goes
 * to row perm[slot] of `out` ([seq_len, heads, 128], any row and head
 * strides), padding slots (perm < 0) are dropped, so the scatter of
 * core/tiling.py:245-252 (scatter_tiles_) happens in the kernel's epilogue.
 * V is in tile order (the v_tiled output of veda_quant_pool_packed).
 * Same bits as veda_sparse_attention followed by veda_scatter_tiles.
 * The caller guarantees that `out` holds seq_len rows at the given strides;
 * slots whose perm entry is at or past seq_len are dropped like padding.
 *   out_heads    [heads] int32, or NULL for heads 0 .. heads - 1: head h of
 *                this call is written to head out_heads[h] of `out` (one
 *                head group of a layer; the caller guarantees every id is
 *                a head of `out`).
 */
int veda_sparse_attention_packed(
    const int8_t* q_i8, const float* q_scale, const int8_t* k_i8,
    const float* k_scale, const void* v, int v_dtype, int64_t v_stride_n,
    int64_t v_stride_h, const int32_t* index, int width, const int32_t* count,
    const int32_t* valid_count, int heads, int n_tiles, void* out,
    int64_t out_stride_n, int64_t out_stride_h, const int64_t* perm,
    int64_t seq_len, const int32_t* out_heads, int32_t* status,
    void* stream);

/*
 * Diagnostic form of veda_sparse_attention for testing its failure path
 * without a GPU fault; it has no counterpart in the reference. Every
 * bounded wait of the kernel gives up after `wait_ns` (0 < wait_ns <= the
 * 2 s the other entry points use), and with `withhold_first_k_load` set the
 * first CTA never issues its first K tile load, so the wait for that tile
 * runs out: the kernel then sets VEDA_STATUS_TIMEOUT in `status`, lets the
 * copies it did issue land, frees its tensor memory and returns, and the
 * device stays usable. With withhold_first_k_load = 0 it computes exactly
 * what veda_sparse_attention computes.
 */
int veda_debug_sparse_attention(
    const int8_t* q_i8, const float* q_scale, const int8_t* k_i8,
    const float* k_scale, const void* v, int v_dtype, int64_t v_stride_n,
    int64_t v_stride_h, const int32_t* index, int width, const int32_t* count,
    const int32_t* valid_count, int heads, int n_tiles, void* out,
    int64_t out_stride_n, int64_t out_stride_h, uint64_t wait_ns,
    int withhold_first_k_load, int32_t* status, void* stream);

/*
 * Tile-order permutation of packed rows (core/tiling.py:227-242,
 * gather_tiles): out[slot, j, :] = x[perm[slot], heads[j], :], and zero
 * where perm[slot] < 0. x is [seq_len, total_heads, 128] 16-bit with
 * strides in elements; out is [n_slots, n_heads, 128] contiguous. Rows or
 * heads out of range read as zero.
 */
int veda_gather_tiles(const void* x, int dtype, int64_t stride_s,
                      int64_t stride_h, int seq_len, int total_heads,
                      const int64_t* perm, int n_slots, const int64_t* heads,
                      int n_heads, void* out, void* stream);

/*
 * Inverse permutation (core/tiling.py:245-252, scatter_tiles_):
 * out[perm[slot], heads[j], :] = tiled[slot, j, :] for real slots; padding
 * slots (and rows or heads out of range) are dropped. out is
 * [seq_len, total_heads, 128] with strides in elements.
 */
int veda_scatter_tiles(const void* tiled, int dtype, const int64_t* perm,
                       int n_slots, const int64_t* heads, int n_heads,
                       int total_heads, void* out, int64_t stride_s,
                       int64_t stride_h, int seq_len, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* VEDA_B200_H_ */
