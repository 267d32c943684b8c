// Kernel (3): block-sparse INT8 attention on tcgen05 tensor cores.
//
// Arithmetic of kernels/sage/sparse_int8.py:136-188 (reference): for each
// (head, query tile) walk the kept key tiles; S = Qi8 . Ki8^T (int32),
// logits = S * q_scale * k_scale (Q was quantised with D^-0.5 * log2(e)
// folded in, so these are base-2 logits); key columns at or past the tile's
// valid count are masked; online softmax with exp2; O += P V; out = O / l.
//
// B200 mapping: a persistent CTA per SM (384 threads, ~177 KB of shared
// memory, all 512 TMEM columns) walks query tiles ("items") one after the
// other. Within a walk the key tiles g are double-buffered in TMEM, so the
// tensor core computes S of tile g + 2 while the softmax works on tile
// g + 1, and each key tile is split into its two 64-key halves, each with
// its own softmax warpgroup, running max, row sum and O accumulator (the
// split-KV form of the online softmax); the halves are merged once per
// walk, O = sum_h O_h 2^(m_h - M) / sum_h l_h 2^(m_h - M), M = max_h m_h.
//   warp 0       TMA producer: the item's Q tile (int8, double buffered
//                across items), then K (int8, 16 KB) and V (16-bit, 32 KB)
//                of each listed key tile into a 3-stage ring, 128-byte
//                swizzled, fetched by tile id.
//   warp 1       P V issuer (and TMEM allocator): O_h(TMEM, f32) (+)=
//                P_h(TMEM) V_h(smem) as 4 x tcgen05.mma kind::f16 (K = 16)
//                per key half h.
//   warp 2       Q K^T issuer: S(TMEM, s32) = Q K^T as 4 x kind::i8
//                (K = 32), once the P V that read the same S buffer is done.
//   warps 4-7    softmax of key half 0, warps 8-11 of key half 1: one query
//                row per thread (TMEM lane = row); load the half row of S,
//                scale, mask, running max with lazy rescaling of O_h (only
//                when the max grows by > 2^8), exp2, write P_h as packed
//                16-bit pairs over the first 32 columns of the half; at the
//                end of a walk, merge the halves and store the row.
// TMEM: S0 [0, 128), S1 [128, 256), O_0 [256, 384), O_1 [384, 512);
// P_h aliases columns [64h, 64h + 32) of S. Every wait is bounded
// (VEDA_STATUS_TIMEOUT) and ends the CTA cleanly.
#include <atomic>

#include "common.cuh"

namespace veda {
namespace {

constexpr int kAttnThreads = 384;
constexpr int kStages = 3;
constexpr uint32_t kQBytes = kTile * kDim;      // int8 Q tile
constexpr uint32_t kKBytes = kTile * kDim;      // int8 K tile
constexpr uint32_t kVBytes = kTile * kDim * 2;  // 16-bit V tile
constexpr uint32_t kSmemQ = 0;                  // 2 Q buffers
constexpr uint32_t kSmemK = kSmemQ + 2 * kQBytes;
constexpr uint32_t kSmemV = kSmemK + kStages * kKBytes;
constexpr uint32_t kSmemXch = kSmemV + kStages * kVBytes;  // [2][2][128] float2
constexpr uint32_t kSmemBar = kSmemXch + 2 * 2 * kTile * 8;
constexpr uint32_t kSmemBytes = kSmemBar + 512;
constexpr uint32_t kTmemCols = 512;
// O is rescaled only when a row's max grows by more than this (log2 units),
// so P stays below 2^8 and the final O / l is unchanged.
constexpr float kRescaleThreshold = 8.0f;
// Register split (setmaxnreg) of the 384 x 168 registers the CTA launches
// with: producer / issuers 128 x 80, softmax 256 x 200 (61440 in all).
constexpr uint32_t kIssueRegs = 80;
constexpr uint32_t kSoftmaxRegs = 200;

__host__ __device__ constexpr uint32_t tmem_s(int b) { return 128u * b; }
__host__ __device__ constexpr uint32_t tmem_o(int h) { return 256u + 128u * h; }

struct Barriers {
  uint64_t q_full[2], q_empty[2];
  uint64_t k_full[kStages], k_empty[kStages];
  uint64_t v_full[kStages], v_empty[kStages];
  uint64_t s_full[2];
  uint64_t p_full[2][2], pv_done[2][2];  // [key half][S buffer]
  uint64_t o_ready, x_full[2], o_free;
  uint64_t fin[2];
  uint32_t tmem_base;
  int abort;
};
static_assert(sizeof(Barriers) <= 512, "barrier block too large");

struct AttnParams {
  const float* q_scale;  // [H][n_tiles]
  const float* k_scale;  // [H][2 n_tiles]
  const int32_t* index;  // [H][n_tiles][width]
  const int32_t* count;  // [H][n_tiles]
  const int32_t* valid;  // [n_tiles]
  void* out;
  int64_t out_sn, out_sh;
  int n_tiles, width, heads;
  int n_items;           // heads * n_tiles
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

// One query tile of one head and its key-tile list.
struct Item {
  int head, qt, count;
  const int32_t* idx;
};

__device__ __forceinline__ Item decode_item(int w, const AttnParams& p) {
  Item it;
  it.head = w / p.n_tiles;
  it.qt = w - it.head * p.n_tiles;
  const int64_t row = static_cast<int64_t>(it.head) * p.n_tiles + it.qt;
  int c = __ldg(p.count + row);
  if (c < 0 || c > p.width) {
    if (threadIdx.x == 0) report(p.status, VEDA_STATUS_BAD_COUNT);
    c = c < 0 ? 0 : p.width;
  }
  it.count = c;
  it.idx = p.index + row * p.width;
  return it;
}

// Items with a non-empty list are numbered n = 0, 1, ... by every role in
// the same order; tiles of those lists are numbered g = 0, 1, ... across
// items. Item n uses Q buffer n % 2; tile g uses S buffer g % 2 and ring
// stage g % 3.

// Warp 0, one thread: the Q tile of each item, then its K / V tiles.
__device__ __forceinline__ void produce(const CUtensorMap* qm, const CUtensorMap* km,
                        const CUtensorMap* vm, uint8_t* smem, Barriers& b,
                        const AttnParams& p) {
  volatile int* abort = &b.abort;
  tma_prefetch(qm);
  tma_prefetch(km);
  tma_prefetch(vm);
  const int n_slots = p.n_tiles * kTile;
  int n = 0, gk = 0, gv = 0;
  bool ok = true;
  for (int w = blockIdx.x; ok && w < p.n_items; w += gridDim.x) {
    const Item it = decode_item(w, p);
    if (it.count == 0) continue;
    ok = mbar_wait(&b.q_empty[n & 1], ((n >> 1) & 1) ^ 1, abort, p.status,
                   VEDA_STATUS_TIMEOUT);
    if (!ok) break;
    mbar_expect_tx(&b.q_full[n & 1], kQBytes);
    tma_load_2d(qm, smem + kSmemQ + (n & 1) * kQBytes, &b.q_full[n & 1], 0,
                it.head * n_slots + it.qt * kTile);
    ++n;
    int t_raw = __ldg(it.idx);
    for (int j = 0; j < it.count && ok; ++j) {
      int t = t_raw;
      if (j + 1 < it.count) t_raw = __ldg(it.idx + j + 1);  // used next step
      if (t < 0 || t >= p.n_tiles) report(p.status, VEDA_STATUS_BAD_INDEX);
      t = clamp_tile(t, p.n_tiles);
      const int stage = gk % kStages;
      const uint32_t ph = (gk / kStages) & 1;
      ok = mbar_wait(&b.k_empty[stage], ph ^ 1, abort, p.status,
                     VEDA_STATUS_TIMEOUT);
      if (!ok) break;
      mbar_expect_tx(&b.k_full[stage], kKBytes);
      tma_load_2d(km, smem + kSmemK + stage * kKBytes, &b.k_full[stage], 0,
                  it.head * n_slots + t * kTile);
      ++gk;
      ok = mbar_wait(&b.v_empty[stage], ph ^ 1, abort, p.status,
                     VEDA_STATUS_TIMEOUT);
      if (!ok) break;
      mbar_expect_tx(&b.v_full[stage], kVBytes);
      uint8_t* vdst = smem + kSmemV + stage * kVBytes;
      tma_load_3d(vm, vdst, &b.v_full[stage], 0, it.head, t * kTile);
      tma_load_3d(vm, vdst + kVBytes / 2, &b.v_full[stage], 64, it.head,
                  t * kTile);
      ++gv;
    }
  }
  // Let every copy this CTA started land before it can exit.
  for (int m = n - 2; m < n; ++m)
    if (m >= 0) drain_wait(&b.q_full[m & 1], (m >> 1) & 1, p.status);
  for (int g = gk - kStages; g < gk; ++g)
    if (g >= 0) drain_wait(&b.k_full[g % kStages], (g / kStages) & 1, p.status);
  for (int g = gv - kStages; g < gv; ++g)
    if (g >= 0) drain_wait(&b.v_full[g % kStages], (g / kStages) & 1, p.status);
}

// Warp 2, one thread: S[g % 2] = Q K^T for every tile g, as soon as its K
// is in and both halves' P V that last read S[g % 2] (tile g - 2) are done.
__device__ __forceinline__ void issue_qk(uint8_t* smem, Barriers& b, uint32_t tmem,
                         const AttnParams& p) {
  volatile int* abort = &b.abort;
  constexpr uint32_t idesc_qk = idesc(2, 1, 0, 128, 128);
  int n = 0, g = 0;
  bool ok = true;
  for (int w = blockIdx.x; ok && w < p.n_items; w += gridDim.x) {
    const Item it = decode_item(w, p);
    if (it.count == 0) continue;
    ok = mbar_wait(&b.q_full[n & 1], (n >> 1) & 1, abort, p.status,
                   VEDA_STATUS_TIMEOUT);
    const uint64_t q_desc =
        smem_desc_sw128(smem_u32(smem + kSmemQ + (n & 1) * kQBytes), 16, 1024);
    for (int j = 0; j < it.count && ok; ++j, ++g) {
      for (int h = 0; h < 2 && ok && g >= 2; ++h)
        ok = mbar_wait(&b.pv_done[h][g & 1], ((g - 2) >> 1) & 1, abort,
                       p.status, VEDA_STATUS_TIMEOUT);
      const int stage = g % kStages;
      if (ok)
        ok = mbar_wait(&b.k_full[stage], (g / kStages) & 1, abort, p.status,
                       VEDA_STATUS_TIMEOUT);
      if (!ok) break;
      tc_fence_after();
      const uint32_t d = tmem + tmem_s(g & 1);
      const uint64_t k_desc =
          smem_desc_sw128(smem_u32(smem + kSmemK + stage * kKBytes), 16, 1024);
      mma_i8_ss(d, q_desc, k_desc, idesc_qk, 0u);
#pragma unroll
      for (int kk = 1; kk < 4; ++kk)  // K = 32 bytes per instruction
        mma_i8_ss(d, q_desc + 2 * kk, k_desc + 2 * kk, idesc_qk, 1u);
      tc_commit(&b.k_empty[stage]);
      tc_commit(&b.s_full[g & 1]);
    }
    if (ok) tc_commit(&b.q_empty[n & 1]);  // the item's last Q K^T
    ++n;
  }
  tc_commit(&b.fin[0]);
  drain_wait(&b.fin[0], 0, p.status);
}

// Warp 1, one thread: O_h (+)= P_h V_h for both key halves of every tile
// g once that half's P is written; the first P V of an item waits until
// the previous item's rows have been read out of O_0 and O_1.
template <typename VT>
__device__ __forceinline__ void issue_pv(uint8_t* smem, Barriers& b, uint32_t tmem,
                         const AttnParams& p) {
  volatile int* abort = &b.abort;
  constexpr uint32_t idesc_pv = idesc(1, Pack<VT>::kFormat, 1, 128, 128);
  int n = 0, g = 0;
  bool ok = true;
  for (int w = blockIdx.x; ok && w < p.n_items; w += gridDim.x) {
    const Item it = decode_item(w, p);
    if (it.count == 0) continue;
    for (int j = 0; j < it.count && ok; ++j, ++g) {
      const int stage = g % kStages;
      for (int h = 0; h < 2 && ok; ++h) {
        ok = mbar_wait(&b.p_full[h][g & 1], (g >> 1) & 1, abort, p.status,
                       VEDA_STATUS_TIMEOUT);
        if (ok && j == 0 && h == 0 && n >= 1)
          ok = mbar_wait(&b.o_free, (n - 1) & 1, abort, p.status,
                         VEDA_STATUS_TIMEOUT);
        if (ok && h == 0)
          ok = mbar_wait(&b.v_full[stage], (g / kStages) & 1, abort, p.status,
                         VEDA_STATUS_TIMEOUT);
        if (!ok) break;
        tc_fence_after();
        const uint32_t o = tmem + tmem_o(h);
        const uint32_t a = tmem + tmem_s(g & 1) + 64 * h;
        const uint64_t v_desc = smem_desc_sw128(
            smem_u32(smem + kSmemV + stage * kVBytes), kVBytes / 2, 1024);
        mma_f16_ts(o, a, v_desc + static_cast<uint64_t>(h * 512), idesc_pv,
                   j > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 1; kk < 4; ++kk)  // 16 keys (8 TMEM columns of P) each
          mma_f16_ts(o, a + 8 * kk,
                     v_desc + static_cast<uint64_t>((4 * h + kk) * 128),
                     idesc_pv, 1u);
        if (h == 1) tc_commit(&b.v_empty[stage]);
        tc_commit(&b.pv_done[h][g & 1]);
      }
    }
    if (ok) tc_commit(&b.o_ready);
    ++n;
  }
  tc_commit(&b.fin[1]);
  drain_wait(&b.fin[1], 0, p.status);
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

// int32 S + 0x4B400000, read as fp32, is exactly 1.5 * 2^23 + S for
// |S| < 2^22 (|S| <= 128 * 127 * 127 here), so S * sc - m comes out of one
// fused multiply-add on the biased value: (1.5 * 2^23 + S) * sc - (off + m).
// The only rounding beyond the reference's fp32 product is that of
// off + m, at most 0.75 units of S, against the ~10^2 units of noise the
// INT8 quantisation itself puts into S.
constexpr uint32_t kMagicBits = 0x4B400000u;
constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23

// Warps 4-7 (key half 0) and 8-11 (key half 1): the softmax of one half of
// every tile of every item, one row per thread; at the end of each walk the
// two halves are merged and each warpgroup stores its 64 output columns.
//
// The global loads that feed a tile (its K scales and valid count, and the
// id of the tile after it) are issued a step ahead and consumed a step
// later, so their latency never sits between two tiles.
template <typename VT>
struct HalfSoftmax {
  Barriers& b;
  const AttnParams& p;
  uint32_t lane_addr, o_self;
  int h, lane;
  // per walk
  const int32_t* idx;
  const float* ks_head;
  float qs;
  int count;
  float m, l;
  // metadata pipeline (raw values, used one step after their load)
  float2 ks_cur, ks_next;
  int valid_cur, valid_next, raw_t1, raw_t2;

  __device__ __forceinline__ bool wait(uint64_t* bar, uint32_t parity) {
    bool ok = mbar_wait(bar, parity, &b.abort, p.status, VEDA_STATUS_TIMEOUT);
    return __all_sync(0xffffffffu, ok);
  }

  __device__ __forceinline__ void load_s(int g, uint32_t* r) {
    const uint32_t a = lane_addr + tmem_s(g & 1) + 64 * h;
    tmem_ld32(a, r);
    tmem_ld32(a + 32, r + 32);
  }

  // One tile: r holds its S (loaded), rn receives the next tile's S.
  __device__ __forceinline__ bool step(int j, int g, uint32_t* r,
                                       uint32_t* rn) {
    const int t1 = clamp_tile(raw_t1, p.n_tiles);
    if (j + 1 < count) {
      ks_next = __ldg(reinterpret_cast<const float2*>(ks_head + 2 * t1));
      valid_next = __ldg(p.valid + t1);
    }
    if (j + 2 < count) raw_t2 = __ldg(idx + j + 2);
    const float sc = qs * (h ? ks_cur.y : ks_cur.x);
    const float off = kMagic * sc;

#pragma unroll
    for (int c = 0; c < 64; ++c) r[c] += kMagicBits;
    if (valid_cur < 64 * h + 64) {
#pragma unroll
      for (int c = 0; c < 64; ++c)
        if (64 * h + c >= valid_cur) r[c] = 0xFF800000u;  // -inf, p = 0
    }
    float ma = -INFINITY, mb = -INFINITY;
#pragma unroll
    for (int c = 0; c < 64; c += 4) {
      ma = max3(ma, __uint_as_float(r[c]), __uint_as_float(r[c + 1]));
      mb = max3(mb, __uint_as_float(r[c + 2]), __uint_as_float(r[c + 3]));
    }
    const float mt = fmaf(fmaxf(ma, mb), sc, -off);  // this half's max logit
    const bool need = mt > m + kRescaleThreshold;
    float alpha = 1.0f;
    if (need) {
      alpha = ex2_approx(m - mt);
      m = mt;
      l *= alpha;
    }
    const uint64_t s2 = f2(sc, sc);
    const float cn = -(off + m);
    const uint64_t n2 = f2(cn, cn);
    uint64_t acc[4] = {0, 0, 0, 0};
    uint32_t pk[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const uint64_t z =
          fma2(f2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1])),
               s2, n2);
      float z0, z1;
      f2_split(z, z0, z1);
      const float p0 = ex2_approx(z0), p1 = ex2_approx(z1);
      acc[i & 3] = add2(acc[i & 3], f2(p0, p1));
      pk[i] = Pack<VT>::two(p0, p1);
    }
    tmem_st32(lane_addr + tmem_s(g & 1) + 64 * h, pk);
    {
      float a0, a1, a2, a3, a4, a5, a6, a7;
      f2_split(acc[0], a0, a1);
      f2_split(acc[1], a2, a3);
      f2_split(acc[2], a4, a5);
      f2_split(acc[3], a6, a7);
      l += ((a0 + a1) + (a2 + a3)) + ((a4 + a5) + (a6 + a7));
    }
    // A grown max rescales O_h, which must first hold this half's P V of
    // the previous tile (rare after the first tiles of a walk).
    if (j > 0 && __any_sync(0xffffffffu, need)) {
      if (!wait(&b.pv_done[h][(g - 1) & 1], ((g - 1) >> 1) & 1)) return false;
      tc_fence_after();
      const uint64_t a2v = f2(alpha, alpha);
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        uint32_t o[32];
        tmem_ld32(o_self + 32 * cc, o);
        tmem_ld_wait(o);
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          float x0, x1;
          f2_split(mul2(f2(__uint_as_float(o[c]), __uint_as_float(o[c + 1])),
                        a2v), x0, x1);
          o[c] = __float_as_uint(x0);
          o[c + 1] = __float_as_uint(x1);
        }
        tmem_st32(o_self + 32 * cc, o);
      }
    }
    tmem_st_wait();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&b.p_full[h][g & 1]);
    if (j + 1 < count) {
      if (!wait(&b.s_full[(g + 1) & 1], ((g + 1) >> 1) & 1)) return false;
      tc_fence_after();
      load_s(g + 1, rn);
      tmem_ld_wait(rn);
      reg_fence32(rn + 32);
    }
    ks_cur = ks_next;
    valid_cur = valid_next;
    raw_t1 = raw_t2;
    return true;
  }
};

template <typename VT>
__device__ __forceinline__ void softmax_loop(int h, uint8_t* smem, Barriers& b, uint32_t tmem,
                             const AttnParams& p, int warp, int lane) {
  const int quarter = warp & 3;  // TMEM lanes this warp may access
  const int row = quarter * 32 + lane;
  HalfSoftmax<VT> sm{b, p};
  sm.lane_addr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
  sm.o_self = sm.lane_addr + tmem_o(h);
  sm.h = h;
  sm.lane = lane;
  const uint32_t o_other = sm.lane_addr + tmem_o(h ^ 1);
  float2* xch = reinterpret_cast<float2*>(smem + kSmemXch);
  int n = 0, g = 0;
  bool good = true;
  for (int w = blockIdx.x; good && w < p.n_items; w += gridDim.x) {
    const Item it = decode_item(w, p);
    VT* out = static_cast<VT*>(p.out) +
              static_cast<int64_t>(it.qt * kTile + row) * p.out_sn +
              static_cast<int64_t>(it.head) * p.out_sh + 64 * h;
    if (it.count == 0) {  // nothing kept: the reference's acc / 1 = 0
#pragma unroll
      for (int c = 0; c < 64; c += 8)
        *reinterpret_cast<uint4*>(out + c) = make_uint4(0, 0, 0, 0);
      continue;
    }
    sm.idx = it.idx;
    sm.count = it.count;
    sm.qs = __ldg(p.q_scale + static_cast<int64_t>(it.head) * p.n_tiles + it.qt);
    sm.ks_head = p.k_scale + static_cast<int64_t>(it.head) * 2 * p.n_tiles;
    const int t0 = clamp_tile(__ldg(it.idx), p.n_tiles);
    sm.ks_cur = __ldg(reinterpret_cast<const float2*>(sm.ks_head + 2 * t0));
    sm.valid_cur = __ldg(p.valid + t0);
    sm.raw_t1 = it.count > 1 ? __ldg(it.idx + 1) : 0;
    sm.ks_next = sm.ks_cur;
    sm.valid_next = sm.valid_cur;
    sm.raw_t2 = 0;
    sm.m = -1e30f;
    sm.l = 0.0f;

    uint32_t r[64];
    good = sm.wait(&b.s_full[g & 1], (g >> 1) & 1);
    if (!good) break;
    tc_fence_after();
    sm.load_s(g, r);
    tmem_ld_wait(r);
    reg_fence32(r + 32);
    for (int j = 0; j < it.count && good; ++j, ++g) good = sm.step(j, g, r, r);
    if (!good) break;
    // Merge the halves: exchange (m, l), then O = sum_h O_h 2^(m_h - M) /
    // sum_h l_h 2^(m_h - M) for this warpgroup's 64 output columns.
    float2* slot = xch + (n & 1) * 2 * kTile;
    slot[h * kTile + row] = make_float2(sm.m, sm.l);
    __syncwarp();
    if (lane == 0) mbar_arrive(&b.x_full[n & 1]);
    good = sm.wait(&b.x_full[n & 1], (n >> 1) & 1) &&
           sm.wait(&b.o_ready, n & 1);
    if (!good) break;
    tc_fence_after();
    const float2 other = slot[(h ^ 1) * kTile + row];
    const float mx = fmaxf(sm.m, other.x);
    const float a_self = ex2_approx(sm.m - mx), a_other = ex2_approx(other.x - mx);
    const float total = sm.l * a_self + other.y * a_other;
    const float inv = total > 0.0f ? 1.0f / total : 1.0f;
    const float w_self = a_self * inv, w_other = a_other * inv;
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      uint32_t os[32], oo[32];
      tmem_ld32(sm.o_self + 64 * h + 32 * cc, os);
      tmem_ld32(o_other + 64 * h + 32 * cc, oo);
      tmem_ld_wait(os);
      reg_fence32(oo);
      float v[32];
#pragma unroll
      for (int c = 0; c < 32; ++c)
        v[c] = __uint_as_float(os[c]) * w_self + __uint_as_float(oo[c]) * w_other;
      store_row<VT>(out + 32 * cc, v);
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&b.o_free);
    ++n;
  }
}

template <uint32_t N>
__device__ __forceinline__ void regs_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void regs_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

template <typename VT>
__global__ void __launch_bounds__(kAttnThreads, 1)
    sparse_attention_kernel(const __grid_constant__ CUtensorMap q_map,
                            const __grid_constant__ CUtensorMap k_map,
                            const __grid_constant__ CUtensorMap v_map,
                            const AttnParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  Barriers& b = *reinterpret_cast<Barriers*>(smem + kSmemBar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    // The 128-byte swizzle pattern assumes 1024-byte aligned tiles.
    b.abort = (smem_u32(smem) & 1023u) != 0 ? 1 : 0;
    if (b.abort) report(p.status, VEDA_STATUS_MISALIGNED);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&b.q_full[i], 1);
      mbar_init(&b.q_empty[i], 1);
      mbar_init(&b.s_full[i], 1);
      mbar_init(&b.x_full[i], 8);
      mbar_init(&b.fin[i], 1);
      for (int h = 0; h < 2; ++h) {
        mbar_init(&b.p_full[h][i], 4);
        mbar_init(&b.pv_done[h][i], 1);
      }
    }
    mbar_init(&b.o_ready, 1);
    mbar_init(&b.o_free, 8);
    for (int st = 0; st < kStages; ++st) {
      mbar_init(&b.k_full[st], 1);
      mbar_init(&b.k_empty[st], 1);
      mbar_init(&b.v_full[st], 1);
      mbar_init(&b.v_empty[st], 1);
    }
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&b.tmem_base, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = b.tmem_base;
  const bool run = b.abort == 0;

  if (warp < 4) {
    regs_dec<kIssueRegs>();
    if (run && lane == 0) {
      if (warp == 0) produce(&q_map, &k_map, &v_map, smem, b, p);
      if (warp == 1) issue_pv<VT>(smem, b, tmem, p);
      if (warp == 2) issue_qk(smem, b, tmem, p);
    }
    __syncwarp();
  } else {
    regs_inc<kSoftmaxRegs>();
    if (run) softmax_loop<VT>((warp - 4) >> 2, smem, b, tmem, p, warp, lane);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

std::atomic<uint32_t> g_smem_set[2][64];
std::atomic<int> g_sm_count[64];

template <typename VT>
int launch(const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm,
           const AttnParams& p, cudaStream_t stream, int dt) {
  const int device = current_device();
  int sms = 148;
  if (device >= 0 && device < 64 && g_sm_count[device].load() > 0) {
    sms = g_sm_count[device].load();
  } else {
    VEDA_CHECK_CUDA(cudaDeviceGetAttribute(
        &sms, cudaDevAttrMultiProcessorCount, device));
    if (device >= 0 && device < 64) g_sm_count[device].store(sms);
  }
  if (device < 0 || device >= 64 || !g_smem_set[dt][device].load()) {
    VEDA_CHECK_CUDA(cudaFuncSetAttribute(
        sparse_attention_kernel<VT>,
        cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
    if (device >= 0 && device < 64) g_smem_set[dt][device].store(1);
  }
  const int grid = p.n_items < sms ? p.n_items : sms;
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
  p.heads = heads;
  p.n_items = heads * n_tiles;
  p.status = status;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (v_dtype == VEDA_BF16) return launch<__nv_bfloat16>(qm, km, vm, p, s, 0);
  return launch<__half>(qm, km, vm, p, s, 1);
}
