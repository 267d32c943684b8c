// Kernel (3): block-sparse INT8 attention on tcgen05 tensor cores.
//
// Arithmetic of kernels/sage/sparse_int8.py:136-188 (reference): for each
// (head, query tile) walk the kept key tiles; S = Qi8 . Ki8^T (int32),
// logits = S * q_scale * k_scale (Q was quantised with D^-0.5 * log2(e)
// folded in, so these are base-2 logits); key columns at or past the tile's
// valid count are masked; online softmax with exp2; O += P V; out = O / l.
//
// B200 mapping, one CTA per (query tile, head), two CTAs per SM:
//   warp 0      TMA producer: the Q tile once, then K (int8, 16 KB) and V
//               (16-bit, 32 KB) of each listed key tile into 2-stage rings,
//               128-byte swizzled, fetched by tile id from the index list.
//   warp 1      TMEM allocator and single-thread MMA issuer:
//               S(TMEM, s32) = Q K^T as 4 x tcgen05.mma kind::i8 (K = 32);
//               O(TMEM, f32) += P(TMEM) V(smem) as 8 x kind::f16 (K = 16).
//   warps 2-5   softmax, one query row per thread (TMEM lane = row): load
//               the S row, scale, mask, running max with lazy rescaling of
//               O (only when the max grows by > 2^8), exp2, write P as
//               packed 16-bit pairs over the first 64 columns of S.
// TMEM: 256 columns per CTA, S in [0, 128), O in [128, 256), P aliases S.
// Every wait is bounded (VEDA_STATUS_TIMEOUT) and ends the CTA cleanly.
#include <atomic>

#include "common.cuh"

namespace veda {
namespace {

constexpr int kAttnThreads = 192;
constexpr uint32_t kQBytes = kTile * kDim;      // int8 Q tile
constexpr uint32_t kKBytes = kTile * kDim;      // int8 K tile
constexpr uint32_t kVBytes = kTile * kDim * 2;  // 16-bit V tile
constexpr uint32_t kSmemQ = 0;
constexpr uint32_t kSmemK = kSmemQ + kQBytes;
constexpr uint32_t kSmemV = kSmemK + 2 * kKBytes;
constexpr uint32_t kSmemBar = kSmemV + 2 * kVBytes;
constexpr uint32_t kSmemBytes = kSmemBar + 256;
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kTmemS = 0;
constexpr uint32_t kTmemO = 128;
// O is rescaled only when a row's max grows by more than this (log2 units),
// so P stays below 2^8 and the final O / l is unchanged.
constexpr float kRescaleThreshold = 8.0f;

struct Barriers {
  uint64_t q_full;
  uint64_t k_full[2], k_empty[2];
  uint64_t v_full[2], v_empty[2];
  uint64_t s_full, p_full, o_full, fin;
  uint32_t tmem_base;
  int abort;
};
static_assert(sizeof(Barriers) <= 256, "barrier block too large");

struct AttnParams {
  const float* q_scale;  // [H][n_tiles]
  const float* k_scale;  // [H][2 n_tiles]
  const int32_t* index;  // [H][n_tiles][width]
  const int32_t* count;  // [H][n_tiles]
  const int32_t* valid;  // [n_tiles]
  void* out;
  int64_t out_sn, out_sh;
  int n_tiles, width;
  int32_t* status;
};

template <typename VT>
struct Pack;
template <>
struct Pack<__nv_bfloat16> {
  static constexpr uint32_t kFormat = 1;
  __device__ static uint32_t two(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
};
template <>
struct Pack<__half> {
  static constexpr uint32_t kFormat = 0;
  __device__ static uint32_t two(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
};

// Bounded wait that ignores the abort flag: used to drain copies and MMAs
// this CTA issued before it exits.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity,
                                           int32_t* status) {
  if (mbar_try_wait(bar, parity)) return;
  const uint64_t start = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_ns() - start > kWaitLimitNs) {
      report(status, VEDA_STATUS_TIMEOUT);
      return;
    }
  }
}

__device__ __forceinline__ int clamp_tile(int t, int n_tiles) {
  return (t < 0 || t >= n_tiles) ? 0 : t;
}

__device__ void produce(const CUtensorMap* qm, const CUtensorMap* km,
                        const CUtensorMap* vm, uint8_t* smem, Barriers& b,
                        const int32_t* idx, int count, int head, int qt,
                        const AttnParams& p) {
  volatile int* abort = &b.abort;
  tma_prefetch(qm);
  tma_prefetch(km);
  tma_prefetch(vm);
  const int n_slots = p.n_tiles * kTile;
  mbar_expect_tx(&b.q_full, kQBytes);
  tma_load_2d(qm, smem + kSmemQ, &b.q_full, 0, head * n_slots + qt * kTile);
  int k_issued = 0, v_issued = 0;
  for (int j = 0; j < count; ++j) {
    int t = __ldg(idx + j);
    if (t < 0 || t >= p.n_tiles) report(p.status, VEDA_STATUS_BAD_INDEX);
    t = clamp_tile(t, p.n_tiles);
    const int s = j & 1;
    const uint32_t ph = (j >> 1) & 1;
    if (!mbar_wait(&b.k_empty[s], ph ^ 1, abort, p.status, VEDA_STATUS_TIMEOUT))
      break;
    mbar_expect_tx(&b.k_full[s], kKBytes);
    tma_load_2d(km, smem + kSmemK + s * kKBytes, &b.k_full[s], 0,
                head * n_slots + t * kTile);
    k_issued = j + 1;
    if (!mbar_wait(&b.v_empty[s], ph ^ 1, abort, p.status, VEDA_STATUS_TIMEOUT))
      break;
    mbar_expect_tx(&b.v_full[s], kVBytes);
    uint8_t* vdst = smem + kSmemV + s * kVBytes;
    tma_load_3d(vm, vdst, &b.v_full[s], 0, head, t * kTile);
    tma_load_3d(vm, vdst + kVBytes / 2, &b.v_full[s], 64, head, t * kTile);
    v_issued = j + 1;
  }
  // Let every copy this CTA started land before it can exit.
  drain_wait(&b.q_full, 0, p.status);
  for (int j = k_issued - 2; j < k_issued; ++j)
    if (j >= 0) drain_wait(&b.k_full[j & 1], (j >> 1) & 1, p.status);
  for (int j = v_issued - 2; j < v_issued; ++j)
    if (j >= 0) drain_wait(&b.v_full[j & 1], (j >> 1) & 1, p.status);
}

__device__ void issue_mma(uint8_t* smem, Barriers& b, uint32_t tmem, int count,
                          uint32_t idesc_pv, const AttnParams& p) {
  volatile int* abort = &b.abort;
  constexpr uint32_t idesc_qk = idesc(2, 1, 0, 128, 128);
  const uint64_t q_desc = smem_desc_sw128(smem_u32(smem + kSmemQ), 16, 1024);
  bool ok = mbar_wait(&b.q_full, 0, abort, p.status, VEDA_STATUS_TIMEOUT);
  for (int j = 0; ok && j < count; ++j) {
    const int s = j & 1;
    const uint32_t ph = (j >> 1) & 1;
    if (!mbar_wait(&b.k_full[s], ph, abort, p.status, VEDA_STATUS_TIMEOUT))
      break;
    // S and P share TMEM: the previous P V must be done before S is rewritten.
    if (j > 0 &&
        !mbar_wait(&b.o_full, (j - 1) & 1, abort, p.status, VEDA_STATUS_TIMEOUT))
      break;
    tc_fence_after();
    const uint64_t k_desc =
        smem_desc_sw128(smem_u32(smem + kSmemK + s * kKBytes), 16, 1024);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk)  // K = 32 bytes per instruction
      mma_i8_ss(tmem + kTmemS, q_desc + 2 * kk, k_desc + 2 * kk, idesc_qk,
                kk > 0 ? 1u : 0u);
    tc_commit(&b.k_empty[s]);
    tc_commit(&b.s_full);
    if (!mbar_wait(&b.p_full, j & 1, abort, p.status, VEDA_STATUS_TIMEOUT))
      break;
    if (!mbar_wait(&b.v_full[s], ph, abort, p.status, VEDA_STATUS_TIMEOUT))
      break;
    tc_fence_after();
    const uint64_t v_desc = smem_desc_sw128(
        smem_u32(smem + kSmemV + s * kVBytes), kVBytes / 2, 1024);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)  // 16 keys (8 TMEM columns of P) each
      mma_f16_ts(tmem + kTmemO, tmem + kTmemS + 8 * kk,
                 v_desc + static_cast<uint64_t>(kk * 128), idesc_pv,
                 (j > 0 || kk > 0) ? 1u : 0u);
    tc_commit(&b.v_empty[s]);
    tc_commit(&b.o_full);
  }
  // Every MMA this CTA issued completes before TMEM is released.
  tc_commit(&b.fin);
  drain_wait(&b.fin, 0, p.status);
}

template <typename VT>
__device__ void store_row(VT* dst, const float* v) {
#pragma unroll
  for (int c = 0; c < 32; c += 8) {
    uint4 u;
    u.x = Pack<VT>::two(v[c], v[c + 1]);
    u.y = Pack<VT>::two(v[c + 2], v[c + 3]);
    u.z = Pack<VT>::two(v[c + 4], v[c + 5]);
    u.w = Pack<VT>::two(v[c + 6], v[c + 7]);
    *reinterpret_cast<uint4*>(dst + c) = u;
  }
}

// Per-tile constants of the softmax: the two K-half scales folded with the
// Q scale, the magic-number offsets that go with them, the valid rows.
struct TileMeta {
  float sc0, sc1;    // q_scale * k_scale of key rows 0-63 / 64-127
  float off0, off1;  // 1.5 * 2^23 * sc0 / sc1
  int valid;
};

// int32 S + 0x4B400000, read as fp32, is exactly 1.5 * 2^23 + S for
// |S| < 2^22 (|S| <= 128 * 127 * 127 here), so S * sc - m comes out of one
// fused multiply-add on the biased value: (1.5 * 2^23 + S) * sc - (off + m).
// The only rounding beyond the reference's fp32 product is that of
// off + m, at most 0.75 units of S, against the ~10^2 units of noise the
// INT8 quantisation itself puts into S.
constexpr uint32_t kMagicBits = 0x4B400000u;
constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23

__device__ __forceinline__ TileMeta load_meta(const float* ks_head,
                                              const int32_t* valid, float qs,
                                              int t) {
  const float2 ks = __ldg(reinterpret_cast<const float2*>(ks_head + 2 * t));
  TileMeta m;
  m.sc0 = qs * ks.x;
  m.sc1 = qs * ks.y;
  m.off0 = kMagic * m.sc0;
  m.off1 = kMagic * m.sc1;
  m.valid = __ldg(valid + t);
  return m;
}

template <typename VT>
__device__ void softmax_rows(Barriers& b, uint32_t tmem, const int32_t* idx,
                             int count, int head, int qt, int warp, int lane,
                             const AttnParams& p) {
  volatile int* abort = &b.abort;
  const int quarter = warp & 3;  // TMEM lanes this warp may access
  const int row = quarter * 32 + lane;
  const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
  const int64_t row_base = static_cast<int64_t>(head) * p.n_tiles + qt;
  const float qs = __ldg(p.q_scale + row_base);
  const float* ks_head = p.k_scale + static_cast<int64_t>(head) * 2 * p.n_tiles;
  VT* out = static_cast<VT*>(p.out) +
            static_cast<int64_t>(qt * kTile + row) * p.out_sn +
            static_cast<int64_t>(head) * p.out_sh;

  // Metadata runs ahead of the walk: tile ids two steps, scales one step,
  // so no global load latency sits between two tiles.
  TileMeta cur = load_meta(ks_head, p.valid, qs,
                           clamp_tile(__ldg(idx), p.n_tiles));
  int t_next = count > 1 ? clamp_tile(__ldg(idx + 1), p.n_tiles) : 0;

  float m = -1e30f, l = 0.0f;
  bool ok = true;
  for (int j = 0; j < count; ++j) {
    TileMeta next = cur;
    int t_after = 0;
    if (j + 1 < count) next = load_meta(ks_head, p.valid, qs, t_next);
    if (j + 2 < count) t_after = clamp_tile(__ldg(idx + j + 2), p.n_tiles);

    ok = mbar_wait(&b.s_full, j & 1, abort, p.status, VEDA_STATUS_TIMEOUT);
    if (!__all_sync(0xffffffffu, ok)) {
      ok = false;
      break;
    }
    tc_fence_after();
    uint32_t r[128];
    tmem_ld32(lane_addr + kTmemS + 0, r);
    tmem_ld32(lane_addr + kTmemS + 32, r + 32);
    tmem_ld32(lane_addr + kTmemS + 64, r + 64);
    tmem_ld32(lane_addr + kTmemS + 96, r + 96);
    tmem_ld_wait(r);
    reg_fence32(r + 32);
    reg_fence32(r + 64);
    reg_fence32(r + 96);
#pragma unroll
    for (int c = 0; c < 128; ++c) r[c] += kMagicBits;
    if (cur.valid < kTile) {
#pragma unroll
      for (int c = 0; c < 128; ++c)
        if (c >= cur.valid) r[c] = 0xFF800000u;  // -inf: never the max, p = 0
    }
    // row max of each 64-column half on the biased values (monotone in S)
    float ma0 = -INFINITY, mb0 = -INFINITY, ma1 = -INFINITY, mb1 = -INFINITY;
#pragma unroll
    for (int c = 0; c < 64; c += 4) {
      ma0 = max3(ma0, __uint_as_float(r[c]), __uint_as_float(r[c + 1]));
      mb0 = max3(mb0, __uint_as_float(r[c + 2]), __uint_as_float(r[c + 3]));
      ma1 = max3(ma1, __uint_as_float(r[c + 64]), __uint_as_float(r[c + 65]));
      mb1 = max3(mb1, __uint_as_float(r[c + 66]), __uint_as_float(r[c + 67]));
    }
    const float mt = fmaxf(fmaf(fmaxf(ma0, mb0), cur.sc0, -cur.off0),
                           fmaf(fmaxf(ma1, mb1), cur.sc1, -cur.off1));
    const bool need = mt > m + kRescaleThreshold;
    float alpha = 1.0f;
    if (need) {
      alpha = ex2_approx(m - mt);
      m = mt;
      l *= alpha;
    }
    const uint64_t s0 = f2(cur.sc0, cur.sc0), s1 = f2(cur.sc1, cur.sc1);
    const float c0 = -(cur.off0 + m), c1 = -(cur.off1 + m);
    const uint64_t n0 = f2(c0, c0), n1 = f2(c1, c1);
    uint64_t acc[4] = {0, 0, 0, 0};
    uint32_t pk[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) {
      const uint64_t z =
          fma2(f2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1])),
               i < 32 ? s0 : s1, i < 32 ? n0 : n1);
      float z0, z1;
      f2_split(z, z0, z1);
      const float p0 = ex2_approx(z0), p1 = ex2_approx(z1);
      acc[i & 3] = add2(acc[i & 3], f2(p0, p1));
      pk[i] = Pack<VT>::two(p0, p1);
    }
    tmem_st32(lane_addr + kTmemS + 0, pk);
    tmem_st32(lane_addr + kTmemS + 32, pk + 32);
    {
      float a0, a1, a2, a3, a4, a5, a6, a7;
      f2_split(acc[0], a0, a1);
      f2_split(acc[1], a2, a3);
      f2_split(acc[2], a4, a5);
      f2_split(acc[3], a6, a7);
      l += ((a0 + a1) + (a2 + a3)) + ((a4 + a5) + (a6 + a7));
    }
    // O (from the previous tiles' P V, complete: the MMA warp waited for it
    // before this tile's Q K^T) is rescaled when some row's max grew.
    if (j > 0 && __any_sync(0xffffffffu, need)) {
      const uint64_t a2v = f2(alpha, alpha);
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        uint32_t o[32];
        tmem_ld32(lane_addr + kTmemO + 32 * cc, o);
        tmem_ld_wait(o);
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          float x0, x1;
          f2_split(mul2(f2(__uint_as_float(o[c]), __uint_as_float(o[c + 1])),
                        a2v), x0, x1);
          o[c] = __float_as_uint(x0);
          o[c + 1] = __float_as_uint(x1);
        }
        tmem_st32(lane_addr + kTmemO + 32 * cc, o);
      }
    }
    tmem_st_wait();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&b.p_full);
    cur = next;
    t_next = t_after;
  }
  if (ok && count > 0)
    ok = mbar_wait(&b.o_full, (count - 1) & 1, abort, p.status,
                   VEDA_STATUS_TIMEOUT);
  if (!__all_sync(0xffffffffu, ok)) return;
  tc_fence_after();
  const float inv = l > 0.0f ? 1.0f / l : 1.0f;
#pragma unroll
  for (int cc = 0; cc < 4; ++cc) {
    uint32_t o[32];
    tmem_ld32(lane_addr + kTmemO + 32 * cc, o);
    tmem_ld_wait(o);
    float v[32];
#pragma unroll
    for (int c = 0; c < 32; ++c) v[c] = __uint_as_float(o[c]) * inv;
    store_row<VT>(out + 32 * cc, v);
  }
}

template <typename VT>
__global__ void __launch_bounds__(kAttnThreads, 2)
    sparse_attention_kernel(const __grid_constant__ CUtensorMap q_map,
                            const __grid_constant__ CUtensorMap k_map,
                            const __grid_constant__ CUtensorMap v_map,
                            const AttnParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  Barriers& b = *reinterpret_cast<Barriers*>(smem + kSmemBar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x, head = blockIdx.y;
  const int64_t row_base = static_cast<int64_t>(head) * p.n_tiles + qt;
  int count = __ldg(p.count + row_base);
  if (count < 0 || count > p.width) {
    if (threadIdx.x == 0) report(p.status, VEDA_STATUS_BAD_COUNT);
    count = count < 0 ? 0 : p.width;
  }
  const int32_t* idx = p.index + row_base * p.width;

  if (threadIdx.x == 0) {
    // The 128-byte swizzle pattern assumes 1024-byte aligned tiles.
    b.abort = (smem_u32(smem) & 1023u) != 0 ? 1 : 0;
    if (b.abort) report(p.status, VEDA_STATUS_MISALIGNED);
    mbar_init(&b.q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&b.k_full[s], 1);
      mbar_init(&b.k_empty[s], 1);
      mbar_init(&b.v_full[s], 1);
      mbar_init(&b.v_empty[s], 1);
    }
    mbar_init(&b.s_full, 1);
    mbar_init(&b.p_full, 4);
    mbar_init(&b.o_full, 1);
    mbar_init(&b.fin, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&b.tmem_base, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = b.tmem_base;
  const bool run = count > 0 && b.abort == 0;

  if (run) {
    if (warp == 0) {
      if (lane == 0)
        produce(&q_map, &k_map, &v_map, smem, b, idx, count, head, qt, p);
      __syncwarp();
    } else if (warp == 1) {
      if (lane == 0)
        issue_mma(smem, b, tmem, count,
                  idesc(1, Pack<VT>::kFormat, 1, 128, 128), p);
      __syncwarp();
    } else {
      softmax_rows<VT>(b, tmem, idx, count, head, qt, warp, lane, p);
    }
  } else if (warp >= 2 && count == 0) {
    const int row = (warp & 3) * 32 + lane;
    VT* out = static_cast<VT*>(p.out) +
              static_cast<int64_t>(qt * kTile + row) * p.out_sn +
              static_cast<int64_t>(head) * p.out_sh;
#pragma unroll
    for (int c = 0; c < kDim; c += 8)
      *reinterpret_cast<uint4*>(out + c) = make_uint4(0, 0, 0, 0);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

std::atomic<uint32_t> g_smem_set[2][64];

template <typename VT>
int launch(const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm,
           const AttnParams& p, int heads, cudaStream_t stream, int dt) {
  const int device = current_device();
  if (device >= 0 && device < 64 && !g_smem_set[dt][device].load()) {
    VEDA_CHECK_CUDA(cudaFuncSetAttribute(
        sparse_attention_kernel<VT>,
        cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
    g_smem_set[dt][device].store(1);
  } else if (device >= 64) {
    VEDA_CHECK_CUDA(cudaFuncSetAttribute(
        sparse_attention_kernel<VT>,
        cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
  }
  dim3 grid(p.n_tiles, heads);
  sparse_attention_kernel<VT><<<grid, kAttnThreads, kSmemBytes, stream>>>(
      qm, km, vm, p);
  VEDA_CHECK_CUDA(cudaGetLastError());
  return VEDA_OK;
}

}  // namespace
}  // namespace veda

using namespace veda;

extern "C" int veda_sparse_attention(
    const int8_t* q_i8, const float* q_scale, const int8_t* k_i8,
    const float* k_scale, const void* v, int v_dtype, int64_t v_stride_n,
    int64_t v_stride_h, const int32_t* index, int width, const int32_t* count,
    const int32_t* valid_count, int heads, int n_tiles, void* out,
    int64_t out_stride_n, int64_t out_stride_h, int32_t* status,
    void* stream) {
  if (int rc = check_device()) return rc;
  if (heads <= 0 || heads > 65535 || n_tiles <= 0 || width <= 0)
    return fail(VEDA_ERR_INVALID, "bad sizes: heads %d, n_tiles %d, width %d",
                heads, n_tiles, width);
  const int64_t n_slots = static_cast<int64_t>(n_tiles) * kTile;
  if (static_cast<int64_t>(heads) * n_slots >= (1ll << 31))
    return fail(VEDA_ERR_INVALID, "heads * slots must stay below 2^31");
  if (v_dtype != VEDA_BF16 && v_dtype != VEDA_F16)
    return fail(VEDA_ERR_INVALID, "v dtype must be bf16 or fp16");
  if (q_i8 == nullptr || k_i8 == nullptr || q_scale == nullptr ||
      k_scale == nullptr || v == nullptr || index == nullptr ||
      count == nullptr || valid_count == nullptr || out == nullptr)
    return fail(VEDA_ERR_INVALID, "null pointer argument");
  if (!aligned16(out) || (out_stride_n * 2) % 16 != 0 ||
      (out_stride_h * 2) % 16 != 0)
    return fail(VEDA_ERR_INVALID, "out rows must be 16-byte aligned");
  CUtensorMap qm, km, vm;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(kDim),
                              static_cast<uint64_t>(heads) * n_slots};
    const uint64_t strides[1] = {static_cast<uint64_t>(kDim)};
    const uint32_t box[2] = {kDim, kTile};
    if (int rc = encode_tiled(&qm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, q_i8,
                              dims, strides, box,
                              CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
    if (int rc = encode_tiled(&km, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, k_i8,
                              dims, strides, box,
                              CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
  }
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(kDim),
                              static_cast<uint64_t>(heads),
                              static_cast<uint64_t>(n_slots)};
    const uint64_t strides[2] = {static_cast<uint64_t>(v_stride_h) * 2,
                                 static_cast<uint64_t>(v_stride_n) * 2};
    const uint32_t box[3] = {64, 1, kTile};
    if (int rc = encode_tiled(
            &vm,
            v_dtype == VEDA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
            3, v, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
  }
  AttnParams p{};
  p.q_scale = q_scale;
  p.k_scale = k_scale;
  p.index = index;
  p.count = count;
  p.valid = valid_count;
  p.out = out;
  p.out_sn = out_stride_n;
  p.out_sh = out_stride_h;
  p.n_tiles = n_tiles;
  p.width = width;
  p.status = status;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (v_dtype == VEDA_BF16)
    return launch<__nv_bfloat16>(qm, km, vm, p, heads, s, 0);
  return launch<__half>(qm, km, vm, p, heads, s, 1);
}
