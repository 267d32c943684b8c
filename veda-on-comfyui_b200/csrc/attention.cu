// Kernel (3): block-sparse INT8 attention on tcgen05 tensor cores.
//
// Arithmetic of kernels/sage/sparse_int8.py:136-188 (reference): for each
// (head, query tile) walk the kept key tiles; S = Qi8 . Ki8^T (int32),
// logits = S * q_scale * k_scale (Q was quantised with D^-0.5 * log2(e)
// folded in, so these are base-2 logits); key columns at or past the tile's
// valid count are masked; online softmax with exp2; O += P V; out = O / l.
//
// B200 mapping: a persistent CTA per SM (384 threads, 225 KB of shared
// memory, all 512 TMEM columns) walks pairs of query tiles of one head, the
// two tiles ("slots" A and B) each with its own key-tile list:
//   warp 0       TMA producer: per pair the two Q tiles (int8, double
//                buffered across pairs), then K (int8, 16 KB) and V
//                (16-bit, 32 KB) of each listed key tile, A and B
//                interleaved, into a 3-stage ring, 128-byte swizzled.
//   warp 1       TMEM allocator and the single MMA-issuing thread, in the
//                fixed order P_A V -> Q_A K' -> P_B V -> Q_B K' ...:
//                S(TMEM, s32) = Q K^T as 4 x tcgen05.mma kind::i8 (K = 32),
//                O(TMEM, f32) += P(TMEM) V(smem) as 8 x kind::f16 (K = 16).
//                While one slot's softmax runs, the tensor core serves the
//                other slot, so exp and MMA overlap.
//   warps 2-3    head-sharded output only: the pushers of slots A and B.
//                They read each finished walk's rows back from this GPU's
//                copy and write them through the NVSwitch multicast
//                address while later walks compute.
//   warps 4-7    softmax of slot A, warps 8-11 of slot B: one query row per
//                thread (TMEM lane = row); load the S row, scale, mask,
//                running max with lazy rescaling of O (only when the max
//                grows by > 2^8; after a walk's first tile the exponentials
//                start at once against the running max and the max is
//                checked on P afterwards), exp2, write P as packed 16-bit
//                pairs over the first 64 columns of S; at the end of a
//                tile's walk, read O out of TMEM (releasing it for the next
//                walk at once), normalise it and store it through a
//                per-warp staging buffer as 64-byte row pieces.
// TMEM: S_A [0, 128), S_B [128, 256), O_A [256, 384), O_B [384, 512); P
// aliases S. One thread issues every MMA and the tensor pipe runs them in
// order, so a Q K^T cannot overwrite P before the P V that reads it, and a
// commit after a Q K^T also covers the P V before it (O is complete
// whenever S is ready). Every wait is bounded (VEDA_STATUS_TIMEOUT).
#include <atomic>

#include "common.cuh"

namespace veda {
namespace {

constexpr int kAttnThreads = 384;
constexpr int kSlots = 2;
constexpr int kStages = 3;
constexpr uint32_t kQBytes = kTile * kDim;      // int8 Q tile
constexpr uint32_t kKBytes = kTile * kDim;      // int8 K tile
constexpr uint32_t kVBytes = kTile * kDim * 2;  // 16-bit V tile
constexpr uint32_t kSmemQ = 0;                  // [slot][buffer] Q tiles
constexpr uint32_t kSmemK = kSmemQ + 4 * kQBytes;
constexpr uint32_t kSmemV = kSmemK + kStages * kKBytes;
// Per softmax warp, 32 rows x 64 bytes: output rows pass through here as
// 32 x 32 boxes on their way to the output as 64-byte row pieces.
constexpr uint32_t kStageBytes = 32 * 64;
constexpr uint32_t kSmemStage = kSmemV + kStages * kVBytes;
constexpr uint32_t kSmemBar = kSmemStage + 8 * kStageBytes;
constexpr uint32_t kSmemBytes = kSmemBar + 512;
static_assert(kSmemBytes <= 227 * 1024, "shared memory over the limit");
constexpr uint32_t kTmemCols = 512;
// O is rescaled only when a row's max grows by more than this (log2 units),
// so P stays below 2^8 and the final O / l is unchanged.
constexpr float kRescaleThreshold = 8.0f;
// Register split (setmaxnreg): the producer / MMA warpgroup gives up
// registers to the two softmax warpgroups. 384 threads launch with 168
// each (64512); 128 x 64 + 256 x 216 = 63488 stays within that.
constexpr uint32_t kLowRegs = 64;
constexpr uint32_t kHighRegs = 216;
// setmaxnreg.inc waits until the registers it asks for are free: a split
// above the launch total (384 threads x 168) would wait forever.
static_assert(128 * kLowRegs + 256 * kHighRegs <= kAttnThreads * 168,
              "register split exceeds the CTA's launch allocation");

__host__ __device__ constexpr uint32_t tmem_s(int slot) { return 128u * slot; }
__host__ __device__ constexpr uint32_t tmem_o(int slot) {
  return 256u + 128u * slot;
}

struct Barriers {
  uint64_t q_full[kSlots][2], q_empty[kSlots][2];
  uint64_t k_full[kStages], k_empty[kStages];
  uint64_t v_full[kStages], v_empty[kStages];
  uint64_t s_full[kSlots], p_full[kSlots];
  uint64_t o_ready[kSlots], o_free[kSlots];
  uint64_t fin;
  uint32_t tmem_base;
  int abort;
  // Head-sharded output: walks whose rows of each (slot, TMEM quarter) are
  // complete in this GPU's copy, for the pusher warps.
  int published[kSlots][4];
};
static_assert(sizeof(Barriers) <= 512, "barrier block too large");

struct AttnParams {
  const float* q_scale;  // [H][n_tiles]
  const float* k_scale;  // [H][2 n_tiles]
  const int32_t* index;  // [H][n_tiles][width]
  const int32_t* count;  // [H][n_tiles]
  const int32_t* valid;  // [n_tiles]
  void* out;
  void* out_mc;          // multicast address of out (element 0), or null
  int64_t out_sn, out_sh;
  // Packed output (null: tile order): slot -> row of `out`, < 0 for
  // padding, which is dropped (core/tiling.py:245-252).
  const int64_t* perm;
  int64_t seq_len;
  // Packed output of one head group (null: all heads): head h of this call
  // is head out_heads[h] of `out`.
  const int32_t* out_heads;
  int n_tiles, width, heads;
  int n_pairs;           // heads * ceil(n_tiles / 2)
  uint64_t wait_ns;      // bound of every wait (kWaitLimitNs in production)
  // Diagnostic only (veda_debug_sparse_attention): CTA 0 never issues its
  // first K load, so the wait for it runs out and the timeout path runs.
  int withhold_first_k;
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

// A pair of query tiles of one head; slot B is absent (qt >= n_tiles) for
// the last pair of a head with an odd tile count.
struct Pair {
  int head;
  int qt[kSlots];
  int count[kSlots];       // kept key tiles, 0 when the slot is absent
  const int32_t* idx[kSlots];
};

__device__ __forceinline__ Pair decode_pair(int w, const AttnParams& p) {
  const int per_head = (p.n_tiles + 1) >> 1;
  Pair pr;
  pr.head = w / per_head;
  const int first = 2 * (w - pr.head * per_head);
#pragma unroll
  for (int s = 0; s < kSlots; ++s) {
    const int qt = first + s;
    pr.qt[s] = qt;
    pr.count[s] = 0;
    pr.idx[s] = nullptr;
    if (qt < p.n_tiles) {
      const int64_t row = static_cast<int64_t>(pr.head) * p.n_tiles + qt;
      int c = __ldg(p.count + row);
      if (c < 0 || c > p.width) {
        if (threadIdx.x == 0) report(p.status, VEDA_STATUS_BAD_COUNT);
        c = c < 0 ? 0 : p.width;
      }
      pr.count[s] = c;
      pr.idx[s] = p.index + row * p.width;
    }
  }
  return pr;
}

// Bounded wait that ignores the abort flag: used to drain copies and MMAs
// this CTA issued before it exits.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity,
                                           const AttnParams& p) {
  if (mbar_try_wait(bar, parity)) return;
  const uint64_t start = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_ns() - start > p.wait_ns) {
      report(p.status, VEDA_STATUS_TIMEOUT);
      return;
    }
  }
}

__device__ __forceinline__ int clamp_tile(int t, int n_tiles) {
  return (t < 0 || t >= n_tiles) ? 0 : t;
}

__device__ __forceinline__ uint8_t* q_tile(uint8_t* smem, int slot, int buf) {
  return smem + kSmemQ + (2 * slot + buf) * kQBytes;
}

// Warp 0: Q tiles per pair, then K / V tiles in the order the MMA thread
// consumes them (A and B interleaved, tile by tile). Lane 0 waits for the
// ring stages and issues the loads; the warp walks the lists with it so the
// outcome of each wait is shared by shuffle.
//
// V is read in tile order, two 64 x 128-row boxes per tile. Reading packed
// V through the permutation here was measured and rejected: the TMA engine
// spends about 65-90 SM clocks per instruction plus about 2.7 clocks per
// 128-byte row, so a 32 KB tile costs ~680 clocks as two tiled boxes but
// ~4,300 as 64 four-row gathers (tile::gather4) and ~1,400 even as 16-row
// boxes, against ~1,100 clocks of attention per tile on a CTA. Packed V is
// copied into tile order by the quantisation pass instead.
__device__ void produce(const CUtensorMap* qm, const CUtensorMap* km,
                        const CUtensorMap* vm, uint8_t* smem, Barriers& b,
                        const AttnParams& p, int lane) {
  volatile int* abort = &b.abort;
  if (lane == 0) {
    tma_prefetch(qm);
    tma_prefetch(km);
    tma_prefetch(vm);
  }
  const int n_slots = p.n_tiles * kTile;
  int q_uses[kSlots][2] = {{0, 0}, {0, 0}};
  int gk = 0, gv = 0;  // K / V tiles issued (ring positions)
  bool ok = true;
  auto from_lane0 = [&](bool v) {
    return __shfl_sync(0xffffffffu, v ? 1 : 0, 0) != 0;
  };
  int it = 0;
  for (int w = blockIdx.x; ok && w < p.n_pairs; w += gridDim.x, ++it) {
    const Pair pr = decode_pair(w, p);
    const int buf = it & 1;
    for (int s = 0; s < kSlots && ok; ++s) {
      if (pr.count[s] == 0) continue;
      if (lane == 0) {
        ok = mbar_wait(&b.q_empty[s][buf], (q_uses[s][buf] & 1) ^ 1, abort,
                       p.status, VEDA_STATUS_TIMEOUT, p.wait_ns);
        if (ok) {
          mbar_expect_tx(&b.q_full[s][buf], kQBytes);
          tma_load_2d(qm, q_tile(smem, s, buf), &b.q_full[s][buf], 0,
                      pr.head * n_slots + pr.qt[s] * kTile);
        }
      }
      ok = from_lane0(ok);
      if (!ok) break;
      ++q_uses[s][buf];
    }
    // Steps (j, s) in issue order: j ascending, both slots per j, a slot
    // skipped once its list is done. The tile id of the next step is loaded
    // one step ahead, so its global load overlaps the waits of the step
    // before instead of following the stage's release.
    const int steps = max(pr.count[0], pr.count[1]);
    int j = 0, s = 0;
    // slot-indexed fields by select, so the pair stays in registers
    auto count_of = [&](int ss) { return ss == 0 ? pr.count[0] : pr.count[1]; };
    auto list_of = [&](int ss) { return ss == 0 ? pr.idx[0] : pr.idx[1]; };
    auto valid = [&](int jj, int ss) { return jj < count_of(ss); };
    auto advance = [&](int& jj, int& ss) {
      do {
        if (++ss == kSlots) { ss = 0; ++jj; }
      } while (jj < steps && !valid(jj, ss));
    };
    if (!valid(j, s)) advance(j, s);
    auto fetch = [&](int jj, int ss) {
      const int t = __ldg(list_of(ss) + jj);
      if (lane == 0 && (t < 0 || t >= p.n_tiles))
        report(p.status, VEDA_STATUS_BAD_INDEX);
      return clamp_tile(t, p.n_tiles);
    };
    int next = j < steps ? fetch(j, s) : 0;
    while (ok && j < steps) {
      const int t = next;
      advance(j, s);
      if (j < steps) next = fetch(j, s);
      const int stage = gk % kStages;
      const uint32_t ph = (gk / kStages) & 1;
      if (lane == 0) {
        ok = mbar_wait(&b.k_empty[stage], ph ^ 1, abort, p.status,
                       VEDA_STATUS_TIMEOUT, p.wait_ns);
        if (ok && !(p.withhold_first_k && blockIdx.x == 0 && gk == 0)) {
          mbar_expect_tx(&b.k_full[stage], kKBytes);
          tma_load_2d(km, smem + kSmemK + stage * kKBytes, &b.k_full[stage],
                      0, pr.head * n_slots + t * kTile);
        }
        if (ok)
          ok = mbar_wait(&b.v_empty[stage], ph ^ 1, abort, p.status,
                         VEDA_STATUS_TIMEOUT, p.wait_ns);
        if (ok) mbar_expect_tx(&b.v_full[stage], kVBytes);
      }
      ok = from_lane0(ok);
      if (!ok) break;
      ++gk;
      if (lane == 0) {
        uint8_t* vdst = smem + kSmemV + stage * kVBytes;
        tma_load_3d(vm, vdst, &b.v_full[stage], 0, pr.head, t * kTile);
        tma_load_3d(vm, vdst + kVBytes / 2, &b.v_full[stage], 64, pr.head,
                    t * kTile);
      }
      ++gv;
    }
  }
  // Let every copy this CTA started land before it can exit.
  if (lane == 0) {
    for (int s = 0; s < kSlots; ++s)
      for (int buf = 0; buf < 2; ++buf)
        if (q_uses[s][buf] > 0)
          drain_wait(&b.q_full[s][buf], (q_uses[s][buf] - 1) & 1, p);
    for (int g = gk - kStages; g < gk; ++g)
      if (g >= 0) drain_wait(&b.k_full[g % kStages], (g / kStages) & 1, p);
    for (int g = gv - kStages; g < gv; ++g)
      if (g >= 0) drain_wait(&b.v_full[g % kStages], (g / kStages) & 1, p);
  }
  __syncwarp();
}

// Warp 1, one thread: every tcgen05.mma of the CTA, in a fixed interleave
// of the two slots.
template <typename VT>
__device__ void issue_mma(uint8_t* smem, Barriers& b, uint32_t tmem,
                          const AttnParams& p) {
  volatile int* abort = &b.abort;
  constexpr uint32_t idesc_qk = idesc(2, 1, 0, 128, 128);
  constexpr uint32_t idesc_pv = idesc(1, Pack<VT>::kFormat, 1, 128, 128);
  int q_uses[kSlots][2] = {{0, 0}, {0, 0}};
  int tiles[kSlots] = {0, 0};  // P tiles taken per slot (p_full phases)
  int items[kSlots] = {0, 0};  // walks finished per slot (o_free phases)
  int gk = 0, gv = 0;          // K / V ring positions
  bool ok = true;

  // The next K / V in the ring has landed (this thread consumes both rings
  // in order, so their parities are unambiguous).
  auto k_ready = [&]() {
    return mbar_wait(&b.k_full[gk % kStages], (gk / kStages) & 1, abort,
                     p.status, VEDA_STATUS_TIMEOUT, p.wait_ns);
  };
  auto v_ready = [&]() {
    return mbar_wait(&b.v_full[gv % kStages], (gv / kStages) & 1, abort,
                     p.status, VEDA_STATUS_TIMEOUT, p.wait_ns);
  };
  // S[s] = Q[s] K^T of the next K in the ring (landed); frees the K stage,
  // signals S.
  auto qk = [&](int s, int buf) {
    const int stage = gk % kStages;
    tc_fence_after();
    const uint64_t q_desc =
        smem_desc_sw128(smem_u32(q_tile(smem, s, buf)), 16, 1024);
    const uint64_t k_desc =
        smem_desc_sw128(smem_u32(smem + kSmemK + stage * kKBytes), 16, 1024);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk)  // K = 32 bytes per instruction
      mma_i8_ss(tmem + tmem_s(s), q_desc + 2 * kk, k_desc + 2 * kk, idesc_qk,
                kk > 0 ? 1u : 0u);
    tc_commit(&b.k_empty[stage]);
    tc_commit(&b.s_full[s]);
    ++gk;
  };
  // O[s] (+)= P[s] V of the next V in the ring (landed); frees the V stage.
  auto pv = [&](int s, bool accumulate) {
    const int stage = gv % kStages;
    tc_fence_after();
    const uint64_t v_desc = smem_desc_sw128(
        smem_u32(smem + kSmemV + stage * kVBytes), kVBytes / 2, 1024);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)  // 16 keys (8 TMEM columns of P) each
      mma_f16_ts(tmem + tmem_o(s), tmem + tmem_s(s) + 8 * kk,
                 v_desc + static_cast<uint64_t>(kk * 128), idesc_pv,
                 (accumulate || kk > 0) ? 1u : 0u);
    tc_commit(&b.v_empty[stage]);
    ++gv;
  };

  int it = 0;
  for (int w = blockIdx.x; ok && w < p.n_pairs; w += gridDim.x, ++it) {
    const Pair pr = decode_pair(w, p);
    const int buf = it & 1;
    for (int s = 0; s < kSlots && ok; ++s) {
      if (pr.count[s] == 0) continue;
      ok = mbar_wait(&b.q_full[s][buf], q_uses[s][buf] & 1, abort, p.status,
                     VEDA_STATUS_TIMEOUT, p.wait_ns);
      ++q_uses[s][buf];
      if (ok) ok = k_ready();
      if (ok) qk(s, buf);
    }
    const int steps = max(pr.count[0], pr.count[1]);
    for (int j = 0; j < steps && ok; ++j) {
      for (int s = 0; s < kSlots && ok; ++s) {
        if (j >= pr.count[s]) continue;
        const bool more = j + 1 < pr.count[s];
        // V of this tile and K of the next are waited for while the
        // softmax still works, so P V and Q K^T follow P without delay.
        ok = v_ready();
        if (ok && more) ok = k_ready();
        if (ok)
          ok = mbar_wait(&b.p_full[s], tiles[s] & 1, abort, p.status,
                         VEDA_STATUS_TIMEOUT, p.wait_ns);
        ++tiles[s];
        // the first P V of a walk overwrites O: the last walk's rows must
        // have been read out of it
        if (ok && j == 0 && items[s] > 0)
          ok = mbar_wait(&b.o_free[s], (items[s] - 1) & 1, abort, p.status,
                         VEDA_STATUS_TIMEOUT, p.wait_ns);
        if (!ok) break;
        pv(s, j > 0);
        if (more) {
          qk(s, buf);
        } else {
          tc_commit(&b.o_ready[s]);
          tc_commit(&b.q_empty[s][buf]);
          ++items[s];
        }
      }
    }
  }
  // Every MMA this CTA issued completes before TMEM is released.
  tc_commit(&b.fin);
  drain_wait(&b.fin, 0, p);
}

// 16 bytes to every GPU bound to the multicast object behind `mc` (one
// store through NVSwitch; the bytes are moved, not interpreted).
__device__ __forceinline__ void store_multicast(void* mc, uint4 u) {
  asm volatile(
      "multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc),
      "f"(__uint_as_float(u.x)), "f"(__uint_as_float(u.y)),
      "f"(__uint_as_float(u.z)), "f"(__uint_as_float(u.w))
      : "memory");
}

// Columns [32 cc, 32 cc + 32) of the warp's 32 rows (v: this lane's row),
// staged in shared memory to turn them around, then written as 64-byte row
// pieces, eight rows per instruction, each to its destination row of `out`
// (dst: element 0 of `out` plus the head offset); rows with dest < 0
// (padding slots) are dropped. dest[i] is the destination row of row
// 8 i + lane / 4 of the warp's 32: the tile-order row itself, or
// perm[slot] for a packed output. Plain stores need no wait before the
// staging buffer is reused (a TMA store of each box would: ~1,000 SM
// clocks a box for the TMA to read it back, measured).
template <typename VT>
__device__ void store_rows(uint8_t* stage, VT* dst, int64_t row_sn,
                           const int64_t* dest, int cc, int lane,
                           const float* v) {
  // 16-byte piece k of row r sits at piece k ^ ((r >> 1) & 3) of the row:
  // the eight rows of a store phase then cover all 32 banks once
  uint4* mine = reinterpret_cast<uint4*>(stage + lane * 64);
  const int sw = (lane >> 1) & 3;
#pragma unroll
  for (int c = 0; c < 32; c += 8) {
    uint4 u;
    u.x = Pack<VT>::two(v[c], v[c + 1]);
    u.y = Pack<VT>::two(v[c + 2], v[c + 3]);
    u.z = Pack<VT>::two(v[c + 4], v[c + 5]);
    u.w = Pack<VT>::two(v[c + 6], v[c + 7]);
    mine[(c / 8) ^ sw] = u;
  }
  __syncwarp();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = 8 * i + (lane >> 2), piece = lane & 3;
    if (dest[i] >= 0) {
      const uint4 u = *reinterpret_cast<const uint4*>(
          stage + r * 64 + (piece ^ ((r >> 1) & 3)) * 16);
      *reinterpret_cast<uint4*>(dst + dest[i] * row_sn + 32 * cc +
                                8 * piece) = u;
    }
  }
  __syncwarp();
}

// Per-tile constants of the softmax: the two K-half scales folded with the
// Q scale, the magic-number offsets that go with them, the valid rows. The
// global loads behind them (K scales, valid count, next tile id) are issued
// a step before the tile that uses them.
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
constexpr float kRescaleFactor = 256.0f;  // 2^kRescaleThreshold
constexpr uint32_t kMagicBits = 0x4B400000u;
constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
constexpr uint32_t kMaskBits = 0xFF800000u - kMagicBits;

// Waits (bounded) until more than `walks` walks are published.
__device__ __forceinline__ bool wait_published(const int* counter, int walks,
                                               volatile int* abort,
                                               int32_t* status,
                                               uint64_t wait_ns) {
  const volatile int* n = counter;
  if (*n <= walks) {
    const uint64_t start = global_ns();
    while (*n <= walks) {
      if (*abort) return false;
      if (global_ns() - start > wait_ns) {
        *abort = 1;
        report(status, VEDA_STATUS_TIMEOUT);
        return false;
      }
      __nanosleep(64);
    }
  }
  __threadfence_block();  // the rows published before the count
  return true;
}

// 16 bytes from global memory through L2 only (rows this CTA's softmax
// warps just stored, behind a fence).
__device__ __forceinline__ uint4 ld_cg_v4(const void* ptr) {
  uint4 u;
  asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(u.x), "=r"(u.y), "=r"(u.z), "=r"(u.w)
               : "l"(ptr));
  return u;
}

// Warps 2 and 3, head-sharded output only: the pusher of slot s. The
// softmax warps write their rows to this GPU's copy of the output and
// publish each walk per TMEM quarter; the pusher reads the
// published rows back (from L2) and writes them through the multicast
// address, so NVSwitch delivers them to every GPU while the next walks
// compute. Rows are never rewritten within a launch, so the pusher may lag.
template <typename VT>
__device__ void push_slot(int s, Barriers& b, const AttnParams& p, int lane) {
  volatile int* abort = &b.abort;
  const char* local = static_cast<const char*>(p.out);
  char* mc = static_cast<char*>(p.out_mc);
  const int64_t row_bytes = p.out_sn * static_cast<int64_t>(sizeof(VT));
  const int64_t head_bytes = p.out_sh * static_cast<int64_t>(sizeof(VT));
  int walks = 0;
  bool ok = true;
  for (int w = blockIdx.x; ok && w < p.n_pairs; w += gridDim.x) {
    const Pair pr = decode_pair(w, p);
    const int qt = pr.qt[s];
    if (qt >= p.n_tiles) continue;
    for (int q = 0; q < 4 && ok; ++q) {
      ok = wait_published(&b.published[s][q], walks, abort, p.status,
                            p.wait_ns);
      if (!ok) break;
      // 32 rows x 256 bytes: lane l moves bytes 16 (l % 16) of rows
      // l / 16, l / 16 + 2, ..., four loads in flight.
      const int64_t first = static_cast<int64_t>(qt * kTile + q * 32 +
                                                 (lane >> 4)) * row_bytes +
                            pr.head * head_bytes + 16 * (lane & 15);
      const int64_t step = 2 * row_bytes;
#pragma unroll
      for (int k0 = 0; k0 < 16; k0 += 4) {
        uint4 u[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
          u[k] = ld_cg_v4(local + first + (k0 + k) * step);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          store_multicast(mc + first + (k0 + k) * step, u[k]);
      }
    }
    ++walks;
  }
  // Multicast rows are ordered before whatever the host does next to
  // signal the other GPUs (a collective on the same stream).
  __threadfence_system();
}

template <typename VT>
__device__ void softmax_loop(int slot, uint8_t* smem, Barriers& b,
                             uint32_t tmem, const AttnParams& p, int warp,
                             int lane) {
  volatile int* abort = &b.abort;
  uint8_t* stage = smem + kSmemStage + (warp - 4) * kStageBytes;
  const int quarter = warp & 3;  // TMEM lanes this warp may access
  const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
  const uint32_t s_addr = lane_addr + tmem_s(slot);
  const uint32_t o_addr = lane_addr + tmem_o(slot);
  int tiles = 0, items = 0;  // phases of s_full / o_ready of this slot
  bool good = true;
  // Head-sharded output: a walk's rows are published to the pusher warp
  // after the warp's stores of them, behind a fence, so the pusher's reads
  // through L2 see them. The publication is put off until the next walk's
  // first S, a pair this slot has no work in, or the end.
  const bool sharded = p.out_mc != nullptr;
  bool unpublished = false;
  auto publish = [&]() {
    if (!unpublished) return;
    __threadfence();
    __syncwarp();
    if (lane == 0) {
      volatile int* n = &b.published[slot][quarter];
      *n = *n + 1;
    }
    __syncwarp();
    unpublished = false;
  };
  for (int w = blockIdx.x; good && w < p.n_pairs; w += gridDim.x) {
    const Pair pr = decode_pair(w, p);
    const int qt = pr.qt[slot];
    if (qt >= p.n_tiles) continue;
    const int count = pr.count[slot];
    const int head = pr.head;
    // the warp's first row (tile order)
    const int row0 = qt * kTile + quarter * 32;
    // the destination rows of this lane's four row pieces: the rows
    // themselves, or through the permutation for a packed output
    int64_t dest[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int row = row0 + 8 * i + (lane >> 2);
      if (p.perm != nullptr) {
        const int64_t d = __ldg(p.perm + row);
        dest[i] = d < p.seq_len ? d : -1;
      } else {
        dest[i] = row;
      }
    }
    const int out_head = p.out_heads != nullptr ? __ldg(p.out_heads + head)
                                                : head;
    VT* dst =
        static_cast<VT*>(p.out) + static_cast<int64_t>(out_head) * p.out_sh;
    if (count == 0) {  // nothing kept: the reference's acc / 1 = 0
      publish();
      float zero[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) zero[c] = 0.0f;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc)
        store_rows<VT>(stage, dst, p.out_sn, dest, cc, lane, zero);
      unpublished = sharded;
      continue;
    }
    const int32_t* idx = pr.idx[slot];
    const float qs = __ldg(p.q_scale + static_cast<int64_t>(head) * p.n_tiles + qt);
    const float* ks_head = p.k_scale + static_cast<int64_t>(head) * 2 * p.n_tiles;
    // Metadata runs ahead of the walk: tile ids two steps, scales one
    // step, so no global load latency sits between two tiles.
    // Raw loads are issued a step before the values are used.
    const int t0 = clamp_tile(__ldg(idx), p.n_tiles);
    float2 ks_cur = __ldg(reinterpret_cast<const float2*>(ks_head + 2 * t0));
    int valid_cur = __ldg(p.valid + t0);
    int raw_t1 = count > 1 ? __ldg(idx + 1) : 0, raw_t2 = 0;
    float2 ks_next = ks_cur;
    int valid_next = valid_cur;

    float m = -1e30f, l = 0.0f;
    for (int j = 0; j < count; ++j) {
      const int t1 = clamp_tile(raw_t1, p.n_tiles);
      if (j + 1 < count) {
        ks_next = __ldg(reinterpret_cast<const float2*>(ks_head + 2 * t1));
        valid_next = __ldg(p.valid + t1);
      }
      if (j + 2 < count) raw_t2 = __ldg(idx + j + 2);
      TileMeta cur;
      cur.sc0 = qs * ks_cur.x;
      cur.sc1 = qs * ks_cur.y;
      cur.off0 = kMagic * cur.sc0;
      cur.off1 = kMagic * cur.sc1;
      cur.valid = valid_cur;

      good = mbar_wait(&b.s_full[slot], tiles & 1, abort, p.status,
                       VEDA_STATUS_TIMEOUT, p.wait_ns);
      ++tiles;
      if (!__all_sync(0xffffffffu, good)) {
        good = false;
        break;
      }
      if (j == 0) publish();
      tc_fence_after();
      uint32_t r[128];
      // S of this tile into registers; masked columns (at or past the
      // tile's valid rows, the same in every lane: a warp-uniform branch)
      // get kMaskBits, which is -inf once the bias is added, so they never
      // win the row max and their exponential is 0.
      auto load_s = [&]() {
        tmem_ld32(s_addr + 0, r);
        tmem_ld32(s_addr + 32, r + 32);
        tmem_ld32(s_addr + 64, r + 64);
        tmem_ld32(s_addr + 96, r + 96);
        tmem_ld_wait(r);
        reg_fence32(r + 32);
        reg_fence32(r + 64);
        reg_fence32(r + 96);
        if (__any_sync(0xffffffffu, cur.valid < kTile)) {
#pragma unroll
          for (int c = 0; c < 128; ++c)
            if (c >= cur.valid) r[c] = kMaskBits;
        }
      };
      // Row max on the biased values (r + kMagicBits read as fp32, monotone
      // in S) of each 64-column half, scaled afterwards; the max grows m
      // only by more than kRescaleThreshold (lazy rescaling of O).
      bool need = false;
      float alpha = 1.0f;
      auto max_pass = [&]() {
        float top0 = -INFINITY, top1 = -INFINITY;
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const float b0 = __uint_as_float(r[2 * i] + kMagicBits);
          const float b1 = __uint_as_float(r[2 * i + 1] + kMagicBits);
          if (i < 32)
            top0 = max3(top0, b0, b1);
          else
            top1 = max3(top1, b0, b1);
        }
        const float mt = fmaxf(fmaf(top0, cur.sc0, -cur.off0),
                               fmaf(top1, cur.sc1, -cur.off1));
        need = mt > m + kRescaleThreshold;
        if (need) {
          alpha = ex2_approx(m - mt);
          m = mt;
          l *= alpha;
        }
      };
      const uint64_t s0 = f2(cur.sc0, cur.sc0), s1 = f2(cur.sc1, cur.sc1);
      uint64_t acc[4];
      uint32_t pk[64];
      float pmax = 0.0f;
      auto exp_pass = [&](auto track) {
        const float c0 = -(cur.off0 + m), c1 = -(cur.off1 + m);
        const uint64_t n0 = f2(c0, c0), n1 = f2(c1, c1);
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[q] = 0;
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const uint64_t z =
              fma2(f2(__uint_as_float(r[2 * i] + kMagicBits),
                      __uint_as_float(r[2 * i + 1] + kMagicBits)),
                   i < 32 ? s0 : s1, i < 32 ? n0 : n1);
          float z0, z1;
          f2_split(z, z0, z1);
          const float p0 = ex2_approx(z0), p1 = ex2_approx(z1);
          acc[i & 3] = add2(acc[i & 3], f2(p0, p1));
          if constexpr (decltype(track)::value) pmax = max3(pmax, p0, p1);
          pk[i] = Pack<VT>::two(p0, p1);
        }
      };
      load_s();
      if (j == 0) {
        // first tile of a walk: the max comes first
        max_pass();
        exp_pass(std::false_type{});
      } else {
        // later tiles: P at once against the running max, the largest P
        // tracked alongside; only if it passes 2^kRescaleThreshold (rare
        // once a walk is under way) is S read again (TMEM still holds it:
        // P is stored over it only below), its max taken and P computed
        // against that. The whole warp redoes it, so no lane keeps its
        // first P beside the reload; a lane whose max held gets the same
        // bits again.
        exp_pass(std::true_type{});
        if (__any_sync(0xffffffffu, pmax > kRescaleFactor)) {
          load_s();
          max_pass();
          exp_pass(std::false_type{});
        }
      }
      tmem_st32(s_addr + 0, pk);
      tmem_st32(s_addr + 32, pk + 32);
      {
        float a0, a1, a2, a3, a4, a5, a6, a7;
        f2_split(acc[0], a0, a1);
        f2_split(acc[1], a2, a3);
        f2_split(acc[2], a4, a5);
        f2_split(acc[3], a6, a7);
        l += ((a0 + a1) + (a2 + a3)) + ((a4 + a5) + (a6 + a7));
      }
      // O holds the P V of every earlier tile of this walk (the commit
      // that signalled S covered them) and is rescaled when a row's max
      // grew.
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        const uint64_t a2v = f2(alpha, alpha);
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          uint32_t o[32];
          tmem_ld32(o_addr + 32 * cc, o);
          tmem_ld_wait(o);
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            float x0, x1;
            f2_split(mul2(f2(__uint_as_float(o[c]), __uint_as_float(o[c + 1])),
                          a2v), x0, x1);
            o[c] = __float_as_uint(x0);
            o[c + 1] = __float_as_uint(x1);
          }
          tmem_st32(o_addr + 32 * cc, o);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&b.p_full[slot]);
      ks_cur = ks_next;
      valid_cur = valid_next;
      raw_t1 = raw_t2;
    }
    if (!good) break;
    good = mbar_wait(&b.o_ready[slot], items & 1, abort, p.status,
                     VEDA_STATUS_TIMEOUT, p.wait_ns);
    ++items;
    if (!__all_sync(0xffffffffu, good)) {
      good = false;
      break;
    }
    tc_fence_after();
    // O comes out of TMEM at once, and the slot's O is released before the
    // stores, so the next walk's first P V does not wait for them.
    uint32_t o[128];
    tmem_ld32(o_addr + 0, o);
    tmem_ld32(o_addr + 32, o + 32);
    tmem_ld32(o_addr + 64, o + 64);
    tmem_ld32(o_addr + 96, o + 96);
    tmem_ld_wait(o);
    reg_fence32(o + 32);
    reg_fence32(o + 64);
    reg_fence32(o + 96);
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&b.o_free[slot]);
    const float inv = l > 0.0f ? 1.0f / l : 1.0f;
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
      float v[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) v[c] = __uint_as_float(o[32 * cc + c]) * inv;
      store_rows<VT>(stage, dst, p.out_sn, dest, cc, lane, v);
    }
    unpublished = sharded;
  }
  if (good) publish();
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
    for (int s = 0; s < kSlots; ++s) {
      for (int buf = 0; buf < 2; ++buf) {
        mbar_init(&b.q_full[s][buf], 1);
        mbar_init(&b.q_empty[s][buf], 1);
      }
      mbar_init(&b.s_full[s], 1);
      mbar_init(&b.p_full[s], 4);
      mbar_init(&b.o_ready[s], 1);
      mbar_init(&b.o_free[s], 4);
    }
    for (int st = 0; st < kStages; ++st) {
      mbar_init(&b.k_full[st], 1);
      mbar_init(&b.k_empty[st], 1);
      mbar_init(&b.v_full[st], 1);
      mbar_init(&b.v_empty[st], 1);
    }
    mbar_init(&b.fin, 1);
    for (int s = 0; s < kSlots; ++s)
      for (int q = 0; q < 4; ++q) b.published[s][q] = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&b.tmem_base, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = b.tmem_base;
  const bool run = b.abort == 0;

  if (warp < 4) {
    regs_dec<kLowRegs>();
    if (run && warp == 0) {
      produce(&q_map, &k_map, &v_map, smem, b, p, lane);
    } else if (run && warp == 1) {
      if (lane == 0) issue_mma<VT>(smem, b, tmem, p);
      __syncwarp();
    } else if (run && warp >= 2 && p.out_mc != nullptr) {
      push_slot<VT>(warp - 2, b, p, lane);
    }
  } else {
    regs_inc<kHighRegs>();
    if (run)
      softmax_loop<VT>((warp - 4) >> 2, smem, b, tmem, p, warp, lane);
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
  const int grid = p.n_pairs < sms ? p.n_pairs : sms;
  sparse_attention_kernel<VT><<<grid, kAttnThreads, kSmemBytes, stream>>>(
      qm, km, vm, p);
  VEDA_CHECK_CUDA(cudaGetLastError());
  return VEDA_OK;
}

}  // namespace
}  // namespace veda

using namespace veda;

namespace {

int attend(const int8_t* q_i8, const float* q_scale, const int8_t* k_i8,
           const float* k_scale, const void* v, int v_dtype,
           int64_t v_stride_n, int64_t v_stride_h, const int32_t* index,
           int width, const int32_t* count, const int32_t* valid_count,
           int heads, int n_tiles, void* out, void* out_mc,
           int64_t out_stride_n, int64_t out_stride_h, int32_t* status,
           void* stream, const int64_t* perm = nullptr, int64_t seq_len = 0,
           const int32_t* out_heads = nullptr,
           uint64_t wait_ns = kWaitLimitNs, int withhold_first_k = 0) {
  if (int rc = check_device()) return rc;
  if (perm != nullptr && (seq_len <= 0 || out_mc != nullptr))
    return fail(VEDA_ERR_INVALID,
                "packed output needs seq_len > 0 and no multicast address");
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
  p.out_mc = out_mc;
  p.out_sn = out_stride_n;
  p.out_sh = out_stride_h;
  p.perm = perm;
  p.seq_len = seq_len;
  p.out_heads = out_heads;
  p.wait_ns = wait_ns;
  p.withhold_first_k = withhold_first_k;
  p.n_tiles = n_tiles;
  p.width = width;
  p.heads = heads;
  p.n_pairs = heads * ((n_tiles + 1) / 2);
  p.status = status;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (v_dtype == VEDA_BF16)
    return launch<__nv_bfloat16>(qm, km, vm, p, s, 0);
  return launch<__half>(qm, km, vm, p, s, 1);
}

}  // namespace

extern "C" int veda_sparse_attention(
    const int8_t* q_i8, const float* q_scale, const int8_t* k_i8,
    const float* k_scale, const void* v, int v_dtype, int64_t v_stride_n,
    int64_t v_stride_h, const int32_t* index, int width, const int32_t* count,
    const int32_t* valid_count, int heads, int n_tiles, void* out,
    int64_t out_stride_n, int64_t out_stride_h, int32_t* status,
    void* stream) {
  return attend(q_i8, q_scale, k_i8, k_scale, v, v_dtype, v_stride_n,
                v_stride_h, index, width, count, valid_count, heads, n_tiles,
                out, nullptr, out_stride_n, out_stride_h, status, stream);
}

extern "C" int veda_sparse_attention_multicast(
    const int8_t* q_i8, const float* q_scale, const int8_t* k_i8,
    const float* k_scale, const void* v, int v_dtype, int64_t v_stride_n,
    int64_t v_stride_h, const int32_t* index, int width, const int32_t* count,
    const int32_t* valid_count, int heads, int n_tiles, void* out,
    void* out_multicast, int64_t out_stride_n, int64_t out_stride_h,
    int32_t* status, void* stream) {
  if (out_multicast == nullptr || !aligned16(out_multicast))
    return fail(VEDA_ERR_INVALID, "out_multicast must be a 16-byte aligned "
                                  "multicast address");
  return attend(q_i8, q_scale, k_i8, k_scale, v, v_dtype, v_stride_n,
                v_stride_h, index, width, count, valid_count, heads, n_tiles,
                out, out_multicast, out_stride_n, out_stride_h, status,
                stream);
}

extern "C" int veda_sparse_attention_packed(
    const int8_t* q_i8, const float* q_scale, const int8_t* k_i8,
    const float* k_scale, const void* v, int v_dtype, int64_t v_stride_n,
    int64_t v_stride_h, const int32_t* index, int width, const int32_t* count,
    const int32_t* valid_count, int heads, int n_tiles, void* out,
    int64_t out_stride_n, int64_t out_stride_h, const int64_t* perm,
    int64_t seq_len, const int32_t* out_heads, int32_t* status,
    void* stream) {
  if (perm == nullptr) return fail(VEDA_ERR_INVALID, "null perm");
  return attend(q_i8, q_scale, k_i8, k_scale, v, v_dtype, v_stride_n,
                v_stride_h, index, width, count, valid_count, heads, n_tiles,
                out, nullptr, out_stride_n, out_stride_h, status, stream, perm,
                seq_len, out_heads);
}

extern "C" int veda_debug_sparse_attention(
    const int8_t* q_i8, const float* q_scale, const int8_t* k_i8,
    const float* k_scale, const void* v, int v_dtype, int64_t v_stride_n,
    int64_t v_stride_h, const int32_t* index, int width, const int32_t* count,
    const int32_t* valid_count, int heads, int n_tiles, void* out,
    int64_t out_stride_n, int64_t out_stride_h, uint64_t wait_ns,
    int withhold_first_k_load, int32_t* status, void* stream) {
  if (wait_ns == 0 || wait_ns > kWaitLimitNs)
    return fail(VEDA_ERR_INVALID, "wait_ns must be in (0, %llu]",
                static_cast<unsigned long long>(kWaitLimitNs));
  return attend(q_i8, q_scale, k_i8, k_scale, v, v_dtype, v_stride_n,
                v_stride_h, index, width, count, valid_count, heads, n_tiles,
                out, nullptr, out_stride_n, out_stride_h, status, stream,
                nullptr, 0, nullptr, wait_ns, withhold_first_k_load ? 1 : 0);
}
