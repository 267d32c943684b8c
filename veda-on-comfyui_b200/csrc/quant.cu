// Kernel (2): per-block INT8 quantisation of Q and K, fused with the
// TripPool features of kernel (1), in one read of each 128-row tile.
//
// Arithmetic of kernels/sage/sparse_int8.py:57-73 (reference): x * pre_scale
// in fp32; scale = max|x| / 127 per (block, head), 1 for an all-zero block;
// q = x / scale; q += 0.5 * sign (>= 0 counts as positive); int8 = trunc(q).
// The quotient is the IEEE-rounded one (see quant8), so the int8 codes
// are bit-exact with an fp32 restatement of those steps.
//
// Pooling follows core/predictor.py:20-60: mean (fp32 sum / max(valid, 1)),
// max and min over the real rows of each video tile, all 0 for an empty tile.
//
// One CTA of 256 threads per (tile, head, tensor); thread t loads 8 rows x 8
// dims with 16-byte vector loads (16 threads cover one 256-byte row).
#include "common.cuh"

namespace veda {
namespace {

constexpr int kQuantThreads = 256;

struct QuantJob {
  const void* x;     // [n_slots, heads, 128] 16-bit
  int8_t* out;       // [heads][n_slots][128]
  float* scale;      // [heads][n_slots / block]
  float* feats;      // [heads][n_video][384] or null
  float pre_scale;
  int block;         // 64 or 128
};

struct QuantParams {
  QuantJob job[2];
  int64_t stride_n, stride_h;  // elements
  int n_tiles;
  int n_heads;                 // output heads of the launch
  const int32_t* valid;        // [n_tiles] or null (all 128)
  int n_video;
  // Packed input (null: rows already in tile order): slot -> packed row,
  // < 0 for padding, which reads as zeros (core/tiling.py:227-242).
  const int64_t* perm;
  int64_t seq_len;
  // Head group (null: all heads): output head h reads input head heads[h],
  // so one head group of a layer is quantised without copying it out.
  const int32_t* heads;
  // Packed V (null: none): CTAs with blockIdx.z == 2 copy V rows through
  // the same permutation and head ids into v_tiled [n_slots, heads, 128]
  // (tile order, contiguous), the operand layout of the attention kernel.
  const void* v;
  int64_t v_stride_n, v_stride_h;  // elements
  void* v_tiled;
};

// Eight 16-bit values of one 16-byte load, widened to fp32 (exact).
__device__ __forceinline__ void unpack8(const uint4& u, float* f,
                                        __nv_bfloat16) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

__device__ __forceinline__ void unpack8(const uint4& u, float* f, __half) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
    f[2 * i] = v.x;
    f[2 * i + 1] = v.y;
  }
}

// Element-wise max / min of two packed pairs of 16-bit values, in their own
// format (the order of the widened fp32 values, exactly), and the packed
// pairs of -inf / +inf that start a running max / min.
__device__ __forceinline__ uint32_t max2(uint32_t a, uint32_t b,
                                         __nv_bfloat16) {
  uint32_t d;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t min2(uint32_t a, uint32_t b,
                                         __nv_bfloat16) {
  uint32_t d;
  asm("min.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t max2(uint32_t a, uint32_t b, __half) {
  uint32_t d;
  asm("max.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t min2(uint32_t a, uint32_t b, __half) {
  uint32_t d;
  asm("min.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// Packed pair whose magnitudes are max(|a|, |b|) element-wise (the sign
// bits come out as the xor of the inputs' and are cleared by the reader).
__device__ __forceinline__ uint32_t absmax2(uint32_t a, uint32_t b,
                                            __nv_bfloat16) {
  uint32_t d;
  asm("max.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t absmax2(uint32_t a, uint32_t b, __half) {
  uint32_t d;
  asm("max.xorsign.abs.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t neg_inf2(__nv_bfloat16) { return 0xFF80FF80u; }
__device__ __forceinline__ uint32_t pos_inf2(__nv_bfloat16) { return 0x7F807F80u; }
__device__ __forceinline__ uint32_t neg_inf2(__half) { return 0xFC00FC00u; }
__device__ __forceinline__ uint32_t pos_inf2(__half) { return 0x7C007C00u; }

// The codes of eight values f: x = RN(f pre), then x / b rounded to
// nearest without a division per element: with y = RN(1 / b), q0 = RN(x y)
// is within one ulp of x / b, the residual r = x - b q0 is exact in one
// FMA, and RN(q0 + r y) = RN(x / b) (Markstein's theorem on FMA-corrected
// division). Only quotients of tiny magnitude (subnormal residuals) can
// differ, and those quantise to 0 either way; the codes are those of an
// IEEE division. Then q += 0.5 with q's sign and truncation (-0 takes
// -0.5 where the reference adds +0.5: both truncate to 0). The fp32 steps
// run two elements at a time; each lane of a packed operation rounds as
// its scalar form.
__device__ __forceinline__ void quant8(const float* f, float pre, float b,
                                       float y, int* c) {
  const uint64_t p2 = f2(pre, pre), nb2 = f2(-b, -b), y2 = f2(y, y);
#pragma unroll
  for (int e = 0; e < 8; e += 2) {
    const uint64_t x = mul2(f2(f[e], f[e + 1]), p2);
    const uint64_t q0 = mul2(x, y2);
    const uint64_t r = fma2(q0, nb2, x);  // x - b q0, exact
    float q[2];
    f2_split(fma2(r, y2, q0), q[0], q[1]);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const float h = __uint_as_float((__float_as_uint(q[k]) & 0x80000000u) |
                                      0x3F000000u);  // 0.5 with q's sign
      c[e + k] = __float2int_rz(__fadd_rn(q[k], h));
    }
  }
}

// The low bytes of four int32 codes, packed in order.
__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
  uint32_t lo, hi, r;
  asm("prmt.b32 %0, %1, %2, 0x0040;" : "=r"(lo) : "r"(a), "r"(b));
  asm("prmt.b32 %0, %1, %2, 0x0040;" : "=r"(hi) : "r"(c), "r"(d));
  asm("prmt.b32 %0, %1, %2, 0x5410;" : "=r"(r) : "r"(lo), "r"(hi));
  return r;
}

// The tile is held as raw 16-bit words (32 registers a thread); the block
// max is taken on them and they are widened once, for the codes. POOL adds
// the TripPool features; their accumulators leave room for few CTAs, so
// the pooling variant reads its tile a second time for the codes (an L2
// hit: the tile was read microseconds earlier by the same CTA) and keeps
// three CTAs per SM. Without pooling a CTA takes HEADS heads of one tile,
// their loads all issued before any arithmetic: one head at four CTAs per
// SM for rows in tile order, two heads (16 row loads in flight per thread)
// for packed rows, whose permutation rows are then read once for both.
template <typename T, bool POOL, int HEADS>
__global__ void __launch_bounds__(kQuantThreads,
                                  POOL ? 3 : (HEADS == 1 ? 4 : 2))
    quant_pool_kernel(const QuantParams p) {
  __shared__ float amax_sh[8][2];
  __shared__ float pool_sh[POOL ? 8 : 1][3][kDim];
  __shared__ float scale_sh[2], inv_sh[2];

  const int tile = blockIdx.x;
  const int n_heads = p.n_heads;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int dc = tid & 15;  // dims 8*dc .. 8*dc+7
  const int rg = tid >> 4;  // rows rg + 16 i
  int head_of[HEADS], src_of[HEADS];
#pragma unroll
  for (int hh = 0; hh < HEADS; ++hh) {
    head_of[hh] = blockIdx.y * HEADS + hh;
    const int h = head_of[hh] < n_heads ? head_of[hh] : n_heads - 1;
    src_of[hh] = p.heads != nullptr ? __ldg(p.heads + h) : h;
  }
  // the tile's rows in the input (the permutation, or the rows themselves)
  int64_t rows[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t slot = static_cast<int64_t>(tile) * kTile + rg + 16 * i;
    rows[i] = p.perm != nullptr ? __ldg(p.perm + slot) : slot;
  }
  auto live_row = [&](int64_t row) {
    return row >= 0 && (p.perm == nullptr || row < p.seq_len);
  };

  if (blockIdx.z == 2) {  // V: a copy into tile order, no arithmetic
    uint4 r[HEADS][8];
#pragma unroll
    for (int hh = 0; hh < HEADS; ++hh) {
      const T* v = static_cast<const T*>(p.v) +
                   static_cast<int64_t>(src_of[hh]) * p.v_stride_h + 8 * dc;
#pragma unroll
      for (int i = 0; i < 8; ++i)
        r[hh][i] = live_row(rows[i])
                       ? __ldg(reinterpret_cast<const uint4*>(
                             v + rows[i] * p.v_stride_n))
                       : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int hh = 0; hh < HEADS; ++hh) {
      if (head_of[hh] >= n_heads) continue;
      T* dst = static_cast<T*>(p.v_tiled) +
               (static_cast<int64_t>(tile) * kTile * n_heads + head_of[hh]) *
                   kDim + 8 * dc;
#pragma unroll
      for (int i = 0; i < 8; ++i)
        *reinterpret_cast<uint4*>(dst + static_cast<int64_t>(rg + 16 * i) *
                                            n_heads * kDim) = r[hh][i];
    }
    return;
  }
  const QuantJob job = blockIdx.z == 0 ? p.job[0] : p.job[1];
  uint4 raw[HEADS][8];
#pragma unroll
  for (int hh = 0; hh < HEADS; ++hh) {
    const T* x = static_cast<const T*>(job.x) +
                 static_cast<int64_t>(src_of[hh]) * p.stride_h + 8 * dc;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      raw[hh][i] = live_row(rows[i])
                       ? __ldg(reinterpret_cast<const uint4*>(
                             x + rows[i] * p.stride_n))
                       : make_uint4(0, 0, 0, 0);
  }
  const float pre = job.pre_scale;
  const int64_t n_slots = static_cast<int64_t>(p.n_tiles) * kTile;

#pragma unroll
  for (int hh = 0; hh < HEADS; ++hh) {
    const int head = head_of[hh];
    if (head >= n_heads) break;  // the same in every thread of the CTA
    if (hh > 0) __syncthreads();  // the last head's reductions are read
    // TripPool over the real rows (a prefix of the tile), before
    // pre-scaling, and max |x * pre| of rows 0-63 (a[0]) and 64-127 (a[1]).
    const bool pool = POOL && job.feats != nullptr && tile < p.n_video;
    const int valid =
        POOL && p.valid != nullptr ? __ldg(p.valid + tile) : kTile;
    // max and min run on the packed 16-bit words (widening is exact and
    // keeps the order), sums in fp32
    float s[8], mx[8], mn[8];
    uint32_t mxw[4], mnw[4];
    if (POOL) {
#pragma unroll
      for (int e = 0; e < 8; ++e) s[e] = 0.0f;
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        mxw[w] = neg_inf2(T());
        mnw[w] = pos_inf2(T());
      }
    }
    // max |x * pre| of rows 0-63 (a[0]) and 64-127 (a[1]): rounding is
    // monotone and symmetric, so it is RN(|pre| * max |x|), and max |x| is
    // taken on the packed 16-bit words (same bits).
    float a[2];
    uint32_t am[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t w[4] = {raw[hh][i].x, raw[hh][i].y, raw[hh][i].z,
                             raw[hh][i].w};
      if (POOL) {
        if (pool && rg + 16 * i < valid) {
          float f[8];
          unpack8(raw[hh][i], f, T());
#pragma unroll
          for (int e = 0; e < 8; ++e) s[e] += f[e];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            mxw[q] = max2(mxw[q], w[q], T());
            mnw[q] = min2(mnw[q], w[q], T());
          }
        }
      }
#pragma unroll
      for (int q = 0; q < 4; ++q)
        am[i >> 2][q] = absmax2(am[i >> 2][q], w[q], T());
    }
    {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t m2 =
            absmax2(absmax2(am[h][0], am[h][1], T()),
                    absmax2(am[h][2], am[h][3], T()), T()) & 0x7FFF7FFFu;
        float mf[8];
        unpack8(make_uint4(m2, 0, 0, 0), mf, T());
        a[h] = __fmul_rn(fmaxf(mf[0], mf[1]), fabsf(pre));
      }
    }
    if (POOL && pool) {
      unpack8(make_uint4(mxw[0], mxw[1], mxw[2], mxw[3]), mx, T());
      unpack8(make_uint4(mnw[0], mnw[1], mnw[2], mnw[3]), mn, T());
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        s[e] += __shfl_xor_sync(0xffffffffu, s[e], 16);
        mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], 16));
        mn[e] = fminf(mn[e], __shfl_xor_sync(0xffffffffu, mn[e], 16));
      }
      if (lane < 16) {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          pool_sh[warp][0][8 * dc + e] = s[e];
          pool_sh[warp][1][8 * dc + e] = mx[e];
          pool_sh[warp][2][8 * dc + e] = mn[e];
        }
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      a[0] = fmaxf(a[0], __shfl_xor_sync(0xffffffffu, a[0], off));
      a[1] = fmaxf(a[1], __shfl_xor_sync(0xffffffffu, a[1], off));
    }
    if (lane == 0) {
      amax_sh[warp][0] = a[0];
      amax_sh[warp][1] = a[1];
    }
    __syncthreads();
    if (tid < 2) {
      float m0 = 0.0f, m1 = 0.0f;
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        m0 = fmaxf(m0, amax_sh[w][0]);
        m1 = fmaxf(m1, amax_sh[w][1]);
      }
      float m = tid == 0 ? m0 : m1;
      if (job.block == kTile) m = fmaxf(m0, m1);
      float sc = __fdiv_rn(m, 127.0f);
      sc = sc > 0.0f ? sc : 1.0f;
      scale_sh[tid] = sc;
      inv_sh[tid] = __frcp_rn(sc);
    }
    if (POOL && pool && tid < kDim) {
      float sum = 0.0f, hi = -INFINITY, lo = INFINITY;
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        sum += pool_sh[w][0][tid];
        hi = fmaxf(hi, pool_sh[w][1][tid]);
        lo = fminf(lo, pool_sh[w][2][tid]);
      }
      float* f = job.feats +
                 (static_cast<int64_t>(head) * p.n_video + tile) * 3 * kDim;
      const bool live = valid > 0;
      f[tid] = live ? __fdiv_rn(sum, static_cast<float>(valid)) : 0.0f;
      f[kDim + tid] = live ? hi : 0.0f;
      f[2 * kDim + tid] = live ? lo : 0.0f;
    }
    __syncthreads();

    const float sc[2] = {scale_sh[0], scale_sh[1]};
    const float inv[2] = {inv_sh[0], inv_sh[1]};
    int8_t* out = job.out + (static_cast<int64_t>(head) * n_slots +
                             static_cast<int64_t>(tile) * kTile) * kDim +
                  8 * dc;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float b = sc[i >> 2], y = inv[i >> 2];
      float f[8];
      if (POOL) {
        const T* x = static_cast<const T*>(job.x) +
                     static_cast<int64_t>(src_of[hh]) * p.stride_h + 8 * dc;
        raw[hh][i] = live_row(rows[i])
                         ? __ldg(reinterpret_cast<const uint4*>(
                               x + rows[i] * p.stride_n))
                         : make_uint4(0, 0, 0, 0);
      }
      unpack8(raw[hh][i], f, T());
      int c[8];
      quant8(f, pre, b, y, c);
      *reinterpret_cast<uint2*>(out + (rg + 16 * i) * kDim) = make_uint2(
          pack4(c[0], c[1], c[2], c[3]), pack4(c[4], c[5], c[6], c[7]));
    }
    if (tid == 0) {
      if (job.block == kTile) {
        job.scale[static_cast<int64_t>(head) * p.n_tiles + tile] = sc[0];
      } else {
        float* sp =
            job.scale + static_cast<int64_t>(head) * 2 * p.n_tiles + 2 * tile;
        sp[0] = sc[0];
        sp[1] = sc[1];
      }
    }
  }
}

int launch_quant(QuantParams p, int n_jobs, int heads, int dtype,
                 cudaStream_t stream) {
  p.n_heads = heads;
  const bool pool = p.job[0].feats != nullptr && p.n_video > 0;
  // two heads per CTA for packed rows without pooling, one otherwise
  const bool two = !pool && p.perm != nullptr;
  const dim3 grid(p.n_tiles, two ? (heads + 1) / 2 : heads, n_jobs);
  if (dtype == VEDA_BF16) {
    if (pool)
      quant_pool_kernel<__nv_bfloat16, true, 1>
          <<<grid, kQuantThreads, 0, stream>>>(p);
    else if (two)
      quant_pool_kernel<__nv_bfloat16, false, 2>
          <<<grid, kQuantThreads, 0, stream>>>(p);
    else
      quant_pool_kernel<__nv_bfloat16, false, 1>
          <<<grid, kQuantThreads, 0, stream>>>(p);
  } else {
    if (pool)
      quant_pool_kernel<__half, true, 1><<<grid, kQuantThreads, 0, stream>>>(p);
    else if (two)
      quant_pool_kernel<__half, false, 2>
          <<<grid, kQuantThreads, 0, stream>>>(p);
    else
      quant_pool_kernel<__half, false, 1>
          <<<grid, kQuantThreads, 0, stream>>>(p);
  }
  VEDA_CHECK_CUDA(cudaGetLastError());
  return VEDA_OK;
}

int check_input(const void* x, int dtype, int64_t stride_n, int64_t stride_h,
                int n_slots, int heads) {
  if (x == nullptr) return fail(VEDA_ERR_INVALID, "null input");
  if (dtype != VEDA_BF16 && dtype != VEDA_F16)
    return fail(VEDA_ERR_INVALID, "input dtype must be bf16 or fp16");
  if (n_slots <= 0 || n_slots % kTile != 0 || heads <= 0)
    return fail(VEDA_ERR_INVALID,
                "n_slots (%d) must be a positive multiple of 128, heads (%d) "
                "positive", n_slots, heads);
  if (n_slots / kTile > 65535 || heads > 65535)
    return fail(VEDA_ERR_INVALID, "too many tiles or heads for one launch");
  if (!aligned16(x) || (stride_n * 2) % 16 != 0 || (stride_h * 2) % 16 != 0)
    return fail(VEDA_ERR_INVALID,
                "input rows must be 16-byte aligned (base, row and head "
                "strides)");
  return VEDA_OK;
}

}  // namespace
}  // namespace veda

using namespace veda;

extern "C" int veda_quantize(const void* x, int dtype, int64_t stride_n,
                             int64_t stride_h, int n_slots, int heads, int dim,
                             int block, float pre_scale, int8_t* out,
                             float* scale, void* stream) {
  if (int rc = check_device()) return rc;
  if (dim != kDim) return fail(VEDA_ERR_INVALID, "head dim must be 128");
  if (block != 64 && block != 128)
    return fail(VEDA_ERR_INVALID, "block must be 64 or 128");
  if (int rc = check_input(x, dtype, stride_n, stride_h, n_slots, heads))
    return rc;
  if (out == nullptr || scale == nullptr || !aligned16(out))
    return fail(VEDA_ERR_INVALID, "null or misaligned output");
  QuantParams p{};
  p.job[0] = QuantJob{x, out, scale, nullptr, pre_scale, block};
  p.stride_n = stride_n;
  p.stride_h = stride_h;
  p.n_tiles = n_slots / kTile;
  p.valid = nullptr;
  p.n_video = 0;
  return launch_quant(p, 1, heads, dtype, static_cast<cudaStream_t>(stream));
}

namespace {

int quant_pool(const void* q, const void* k, int dtype, int64_t stride_n,
               int64_t stride_h, int n_slots, int heads,
               const int32_t* valid_count, int n_video_tiles,
               float q_pre_scale, int8_t* q_i8, float* q_scale, int8_t* k_i8,
               float* k_scale, float* feats_q, float* feats_k,
               const int64_t* perm, int64_t seq_len, const int32_t* head_ids,
               void* stream, const void* v = nullptr, int64_t v_stride_n = 0,
               int64_t v_stride_h = 0, void* v_tiled = nullptr) {
  if (int rc = check_device()) return rc;
  // packed inputs have seq_len rows; the check wants a whole number of tiles
  const int rows = perm == nullptr ? n_slots : kTile;
  if (int rc = check_input(q, dtype, stride_n, stride_h, rows, heads))
    return rc;
  if (int rc = check_input(k, dtype, stride_n, stride_h, rows, heads))
    return rc;
  if (n_slots <= 0 || n_slots % kTile != 0 || n_slots / kTile > 65535)
    return fail(VEDA_ERR_INVALID,
                "slots must be a positive whole number of tiles (at most "
                "65535)");
  if (perm != nullptr && seq_len <= 0)
    return fail(VEDA_ERR_INVALID, "packed input needs seq_len > 0");
  if (q_i8 == nullptr || k_i8 == nullptr || q_scale == nullptr ||
      k_scale == nullptr || !aligned16(q_i8) || !aligned16(k_i8))
    return fail(VEDA_ERR_INVALID, "null or misaligned output");
  const int n_tiles = n_slots / kTile;
  if ((feats_q != nullptr) != (feats_k != nullptr))
    return fail(VEDA_ERR_INVALID, "feats_q and feats_k go together");
  if (feats_q != nullptr &&
      (valid_count == nullptr || n_video_tiles < 0 || n_video_tiles > n_tiles))
    return fail(VEDA_ERR_INVALID,
                "pooling needs valid_count and 0 <= n_video_tiles <= n_tiles");
  QuantParams p{};
  p.job[0] = QuantJob{q, q_i8, q_scale, feats_q, q_pre_scale, kTile};
  p.job[1] = QuantJob{k, k_i8, k_scale, feats_k, 1.0f, kKeyBlock};
  p.stride_n = stride_n;
  p.stride_h = stride_h;
  p.n_tiles = n_tiles;
  p.valid = valid_count;
  p.n_video = feats_q != nullptr ? n_video_tiles : 0;
  p.perm = perm;
  p.seq_len = seq_len;
  p.heads = head_ids;
  if ((v == nullptr) != (v_tiled == nullptr))
    return fail(VEDA_ERR_INVALID, "v and v_tiled go together");
  if (v != nullptr) {
    if (perm == nullptr)
      return fail(VEDA_ERR_INVALID, "a V copy needs packed input (perm)");
    if (int rc = check_input(v, dtype, v_stride_n, v_stride_h, kTile, heads))
      return rc;
    if (!aligned16(v_tiled))
      return fail(VEDA_ERR_INVALID, "v_tiled must be 16-byte aligned");
    p.v = v;
    p.v_stride_n = v_stride_n;
    p.v_stride_h = v_stride_h;
    p.v_tiled = v_tiled;
  }
  return launch_quant(p, v != nullptr ? 3 : 2, heads, dtype,
                      static_cast<cudaStream_t>(stream));
}

}  // namespace

extern "C" int veda_quant_pool(const void* q, const void* k, int dtype,
                               int64_t stride_n, int64_t stride_h, int n_slots,
                               int heads, const int32_t* valid_count,
                               int n_video_tiles, float q_pre_scale,
                               int8_t* q_i8, float* q_scale, int8_t* k_i8,
                               float* k_scale, float* feats_q, float* feats_k,
                               void* stream) {
  return quant_pool(q, k, dtype, stride_n, stride_h, n_slots, heads,
                    valid_count, n_video_tiles, q_pre_scale, q_i8, q_scale,
                    k_i8, k_scale, feats_q, feats_k, nullptr, 0, nullptr,
                    stream);
}

extern "C" int veda_quant_pool_packed(
    const void* q, const void* k, int dtype, int64_t stride_n,
    int64_t stride_h, int64_t seq_len, const int64_t* perm, int n_slots,
    int heads, const int32_t* valid_count, int n_video_tiles,
    float q_pre_scale, int8_t* q_i8, float* q_scale, int8_t* k_i8,
    float* k_scale, float* feats_q, float* feats_k, const void* v,
    int64_t v_stride_n, int64_t v_stride_h, void* v_tiled,
    const int32_t* head_ids, void* stream) {
  if (perm == nullptr) return fail(VEDA_ERR_INVALID, "null perm");
  return quant_pool(q, k, dtype, stride_n, stride_h, n_slots, heads,
                    valid_count, n_video_tiles, q_pre_scale, q_i8, q_scale,
                    k_i8, k_scale, feats_q, feats_k, perm, seq_len, head_ids,
                    stream, v, v_stride_n, v_stride_h, v_tiled);
}
