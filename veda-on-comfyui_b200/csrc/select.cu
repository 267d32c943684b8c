// Kernel (1c): Veda top-k key-tile selection written straight into compact,
// ascending index lists, one warp per (head, query tile).
//
// Rules of core/selection.py:132-227 (reference): within each sparse column
// block a row's empty tiles score -inf and its own tile +inf; the row keeps
// the k_lo + extra[row] highest scores that are > -inf (torch.topk then a
// prefix of the sorted values). Keep-all blocks, global columns and global
// rows keep every non-empty tile. The kept set is then ANDed with kv_ok
// (backends/triton_int8.py:51) and listed in ascending tile order.
//
// The k-th largest score is found exactly with a bitwise radix search on
// order-preserving uint32 keys (warp ballots and reductions, no sort); ties
// at the threshold are taken in ascending tile order. The list is written
// with ballot-prefix compaction in ascending column order, so it needs no
// sort either.
#include "common.cuh"

namespace veda {
namespace {

constexpr int kSelectWarps = 8;
constexpr uint32_t kFull = 0xffffffffu;

struct SelectParams {
  const float* scores;
  int64_t stride_h, stride_r;
  int heads, n_video, n_tiles;
  const uint8_t* kv_ok;
  int n_blocks;
  veda_column_block blocks[2];
  const uint8_t* extra;
  const uint8_t* mask;  // mask_to_index only
  int width;
  int32_t* index;
  int32_t* count;
  int32_t* status;
};

// Order-preserving map of fp32 bit patterns onto uint32.
__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

constexpr uint32_t kNegInfKey = 0x007FFFFFu;  // order_key(-inf)

// Warp-cooperative ascending emitter of kept column ids.
struct Emitter {
  int32_t* out;
  int width;
  int n;  // warp-uniform count so far

  __device__ __forceinline__ void push(bool keep, int col, int lane) {
    const uint32_t ballot = __ballot_sync(kFull, keep);
    const int pos = n + __popc(ballot & ((1u << lane) - 1u));
    if (keep && pos < width) out[pos] = col;
    n += __popc(ballot);
  }
};

__device__ void emit_kv_ok(Emitter& em, const uint8_t* kv_ok, int lo, int hi,
                           int lane) {
  for (int c0 = lo; c0 < hi; c0 += 32) {
    const int c = c0 + lane;
    const bool keep = c < hi && __ldg(kv_ok + c) != 0;
    em.push(keep, c, lane);
  }
}

template <int VPL>
__device__ void emit_topk(Emitter& em, const SelectParams& p,
                          const float* row_scores, int row, int start,
                          int stop, int kk, int lane) {
  uint32_t key[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = start + 32 * i + lane;
    key[i] = 0;
    if (c < stop) {
      float s = __ldg(row_scores + c);
      if (__ldg(p.kv_ok + c) == 0) s = -INFINITY;
      if (c == row) s = INFINITY;
      key[i] = order_key(s);
    }
  }
  const int n_cols = stop - start;
  uint32_t thresh = 0;
  if (kk < n_cols) {
    // Largest T with |{key >= T}| >= kk: the kk-th largest key. The search
    // stops early once exactly kk keys are >= T: those are the kk largest,
    // and the selection below (every key > T, then keys == T) keeps exactly
    // them, as it would with the exact kk-th largest key.
#pragma unroll 1
    for (int bit = 31; bit >= 0; --bit) {
      const uint32_t cand = thresh | (1u << bit);
      int cnt = 0;
#pragma unroll
      for (int i = 0; i < VPL; ++i)
        cnt += (start + 32 * i + lane < stop && key[i] >= cand) ? 1 : 0;
      cnt = __reduce_add_sync(kFull, cnt);
      if (cnt >= kk) thresh = cand;
      if (cnt == kk) break;  // warp-uniform
    }
  }
  int above = 0;
#pragma unroll
  for (int i = 0; i < VPL; ++i)
    above += (start + 32 * i + lane < stop && key[i] > thresh) ? 1 : 0;
  above = __reduce_add_sync(kFull, above);
  const int need_eq = kk < n_cols ? kk - above : n_cols;
  int eq_seen = 0;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = start + 32 * i + lane;
    if (start + 32 * i >= stop) break;
    const bool in = c < stop;
    const bool eq = in && key[i] == thresh;
    const uint32_t eq_ballot = __ballot_sync(kFull, eq);
    const int eq_rank = eq_seen + __popc(eq_ballot & ((1u << lane) - 1u));
    eq_seen += __popc(eq_ballot);
    bool keep = in && key[i] != kNegInfKey &&
                (key[i] > thresh || (eq && eq_rank < need_eq));
    if (kk >= n_cols) keep = in && key[i] != kNegInfKey;
    keep = keep && __ldg(p.kv_ok + c) != 0;
    em.push(keep, c, lane);
  }
}

template <int VPL>
__global__ void __launch_bounds__(kSelectWarps * 32)
    select_kernel(const SelectParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kSelectWarps + warp;
  const int head = blockIdx.y;
  if (row >= p.n_tiles) return;
  Emitter em{p.index + (static_cast<int64_t>(head) * p.n_tiles + row) * p.width,
             p.width, 0};
  if (p.mask != nullptr) {
    const uint8_t* m = p.mask + (static_cast<int64_t>(head) * p.n_tiles + row) *
                                    p.n_tiles;
    for (int c0 = 0; c0 < p.n_tiles; c0 += 32) {
      const int c = c0 + lane;
      const bool keep =
          c < p.n_tiles && __ldg(m + c) != 0 && __ldg(p.kv_ok + c) != 0;
      em.push(keep, c, lane);
    }
  } else if (row >= p.n_video) {
    emit_kv_ok(em, p.kv_ok, 0, p.n_tiles, lane);
  } else {
    const float* row_scores =
        p.scores + head * p.stride_h + static_cast<int64_t>(row) * p.stride_r;
    for (int b = 0; b < p.n_blocks; ++b) {
      const veda_column_block blk = p.blocks[b];
      if (blk.keeps_all) {
        emit_kv_ok(em, p.kv_ok, blk.start, blk.stop, lane);
      } else {
        const int kk = blk.k_lo + (__ldg(p.extra + b * p.n_video + row) ? 1 : 0);
        emit_topk<VPL>(em, p, row_scores, row, blk.start, blk.stop, kk, lane);
      }
    }
    emit_kv_ok(em, p.kv_ok, p.n_video, p.n_tiles, lane);
  }
  int32_t* out = em.out;
  for (int c = em.n + lane; c < p.width; c += 32) out[c] = -1;
  if (lane == 0) {
    if (em.n > p.width) report(p.status, VEDA_STATUS_OVERFLOW);
    p.count[static_cast<int64_t>(head) * p.n_tiles + row] =
        em.n < p.width ? em.n : p.width;
  }
}

int launch_select(const SelectParams& p, int max_cols, cudaStream_t stream) {
  dim3 grid((p.n_tiles + kSelectWarps - 1) / kSelectWarps, p.heads);
  dim3 block(kSelectWarps * 32);
  const int vpl = (max_cols + 31) / 32;
  if (vpl <= 1)
    select_kernel<1><<<grid, block, 0, stream>>>(p);
  else if (vpl <= 2)
    select_kernel<2><<<grid, block, 0, stream>>>(p);
  else if (vpl <= 4)
    select_kernel<4><<<grid, block, 0, stream>>>(p);
  else if (vpl <= 8)
    select_kernel<8><<<grid, block, 0, stream>>>(p);
  else if (vpl <= 16)
    select_kernel<16><<<grid, block, 0, stream>>>(p);
  else if (vpl <= 32)
    select_kernel<32><<<grid, block, 0, stream>>>(p);
  else
    select_kernel<64><<<grid, block, 0, stream>>>(p);
  VEDA_CHECK_CUDA(cudaGetLastError());
  return VEDA_OK;
}

}  // namespace
}  // namespace veda

using namespace veda;

extern "C" int veda_select(const float* scores, int64_t score_stride_h,
                           int64_t score_stride_r, int heads, int n_video,
                           int n_tiles, const uint8_t* kv_ok, int n_blocks,
                           const veda_column_block* blocks,
                           const uint8_t* extra, int width, int32_t* index,
                           int32_t* count, int32_t* status, void* stream) {
  if (int rc = check_device()) return rc;
  if (heads <= 0 || heads > 65535 || n_tiles <= 0 || n_video < 0 ||
      n_video > n_tiles || width <= 0)
    return fail(VEDA_ERR_INVALID,
                "bad sizes: heads %d, n_video %d, n_tiles %d, width %d", heads,
                n_video, n_tiles, width);
  if (kv_ok == nullptr || index == nullptr || count == nullptr)
    return fail(VEDA_ERR_INVALID, "null kv_ok / index / count");
  if (n_blocks < 0 || n_blocks > 2 || (n_video > 0 && n_blocks == 0))
    return fail(VEDA_ERR_INVALID, "n_blocks must be 1 or 2");
  SelectParams p{};
  int max_cols = 1, prev = 0;
  bool sparse = false;
  for (int b = 0; b < n_blocks; ++b) {
    const veda_column_block blk = blocks[b];
    if (blk.start != prev || blk.stop <= blk.start || blk.stop > n_video)
      return fail(VEDA_ERR_INVALID,
                  "column blocks must tile [0, n_video) in order");
    prev = blk.stop;
    if (!blk.keeps_all) {
      if (blk.k_lo < 1 || blk.k_lo > blk.stop - blk.start)
        return fail(VEDA_ERR_INVALID, "k_lo %d outside [1, %d]", blk.k_lo,
                    blk.stop - blk.start);
      sparse = true;
      max_cols = blk.stop - blk.start > max_cols ? blk.stop - blk.start
                                                 : max_cols;
    }
    p.blocks[b] = blk;
  }
  if (n_blocks > 0 && prev != n_video)
    return fail(VEDA_ERR_INVALID, "column blocks must end at n_video");
  if (max_cols > 2048)
    return fail(VEDA_ERR_INVALID, "a column block wider than 2048 tiles");
  if (sparse && (scores == nullptr || extra == nullptr))
    return fail(VEDA_ERR_INVALID, "sparse blocks need scores and extra");
  p.scores = scores;
  p.stride_h = score_stride_h;
  p.stride_r = score_stride_r;
  p.heads = heads;
  p.n_video = n_video;
  p.n_tiles = n_tiles;
  p.kv_ok = kv_ok;
  p.n_blocks = n_blocks;
  p.extra = extra;
  p.mask = nullptr;
  p.width = width;
  p.index = index;
  p.count = count;
  p.status = status;
  return launch_select(p, max_cols, static_cast<cudaStream_t>(stream));
}

extern "C" int veda_mask_to_index(const uint8_t* mask, const uint8_t* kv_ok,
                                  int heads, int n_tiles, int width,
                                  int32_t* index, int32_t* count,
                                  int32_t* status, void* stream) {
  if (int rc = check_device()) return rc;
  if (heads <= 0 || heads > 65535 || n_tiles <= 0 || width <= 0)
    return fail(VEDA_ERR_INVALID, "bad sizes: heads %d, n_tiles %d, width %d",
                heads, n_tiles, width);
  if (mask == nullptr || kv_ok == nullptr || index == nullptr ||
      count == nullptr)
    return fail(VEDA_ERR_INVALID, "null mask / kv_ok / index / count");
  SelectParams p{};
  p.heads = heads;
  p.n_video = 0;
  p.n_tiles = n_tiles;
  p.kv_ok = kv_ok;
  p.mask = mask;
  p.width = width;
  p.index = index;
  p.count = count;
  p.status = status;
  return launch_select(p, 1, static_cast<cudaStream_t>(stream));
}
