// INT8 flash attention for sm_100a: int8 Q.K^T on tcgen05 (kind::i8, int32 S in TMEM), fp32
// online softmax (one thread owns one query row, so row max and row sum are thread-local),
// bf16/fp16 P written back to TMEM, and P.V on tcgen05 (kind::f16, fp32 O in TMEM).
//
// Two quantization modes share the main kernel:
//   kModeRef      the reference's scheme (src/diffucore/kernels/int8_attn_sm80.cu):
//                 Q per token, K per 64-key block after subtracting K's per-channel mean.
//   kModeBlock64  Q and K both per 64-token block, no mean (symmetric abs-max).
// The prep kernels write contiguous int8 codes + fp32 scales into the caller's workspace; the
// main kernel TMA-loads them. V is read in place from the caller's (B, L, H, D) strides.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>
#include "sm100.cuh"
#include "quant.cuh"

namespace dc {

enum AttnMode : int { kModeRef = 0, kModeBlock64 = 1 };

constexpr int kAttnBM = 128;        // query rows per Q tile (one softmax warpgroup)
constexpr int kAttnBN = 128;        // keys per K/V tile
constexpr int kAttnKBlk = 64;       // keys per K scale block
constexpr int kAttnRows = 256;      // query rows per CTA (two Q tiles)
constexpr int kAttnThreads = 320;   // warps 0-7 softmax (2 x 4), warp 8 TMA, warp 9 MMA
constexpr int kAttnStages = 3;
constexpr int kStatWin = 128;       // rows per K-sum window (the reference's FLUSH_EVERY * BC)

// ----------------------------------------------------------------------------- prep

// Per-(b, h, window) partial K column sums in the reference's fixed order
// (int8_attn_sm80.cu:92-135): thread (rg, ch) adds rows r0+rg, r0+rg+16, ... of its 8 channels;
// the 16 row-group partials are then added in order rg = 0..15. Six CTAs per SM, so that the
// windows x heads of a 4608-token, 24-head call run in one wave.
template <typename T, int D>
__global__ void __launch_bounds__(16 * (D / 8), 6)
k_stats_kernel(const T* __restrict__ k, float* __restrict__ kpart, int L, int H, int64_t sb, int64_t sl,
               int64_t sh) {
  constexpr int NCH = D / 8;
  const int b = blockIdx.z, h = blockIdx.y;
  const int ch = threadIdx.x % NCH, rg = threadIdx.x / NCH;
  const T* kb = k + b * sb + h * sh + ch * 8;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  const int r0 = blockIdx.x * kStatWin, r1 = min(L, r0 + kStatWin);
  for (int r = r0 + rg; r < r1; r += 16) {
    float f[8];
    Vec8<T>::load(kb + r * sl, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = __fadd_rn(acc[i], f[i]);
  }
  __shared__ float red[16][D + 1];
#pragma unroll
  for (int i = 0; i < 8; ++i) red[rg][ch * 8 + i] = acc[i];
  __syncthreads();
  if (threadIdx.x < D) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) s = __fadd_rn(s, red[i][threadIdx.x]);
    kpart[(static_cast<int64_t>(b * H + h) * gridDim.x + blockIdx.x) * D + threadIdx.x] = s;
  }
}

// ksum[bh, d] = sum over windows in order (int8_attn_sm80.cu:137-142); the partials are loaded
// eight at a time ahead of the in-order adds.
template <int D>
__global__ void k_sum_kernel(const float* __restrict__ kpart, float* __restrict__ ksum, int nwin) {
  const float* src = kpart + static_cast<int64_t>(blockIdx.x) * nwin * D + threadIdx.x;
  float s = 0.f;
  for (int w0 = 0; w0 < nwin; w0 += 8) {
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = w0 + i < nwin ? src[(w0 + i) * D] : 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (w0 + i < nwin) s = __fadd_rn(s, v[i]);
  }
  ksum[blockIdx.x * D + threadIdx.x] = s;
}

// Per-64-row block int8 codes: x' = x - ksum * (1/L) (as one fused multiply-add, the form the
// reference's `f.x - ksum[..] * inv_l` takes under nvcc's default contraction,
// int8_attn_sm80.cu:57-58) when `ksum` is given, else x' = x; amax over the 64 x D block;
// scale = amax / 127; code = rn(x' * (127 / amax)), 0 when amax == 0 (:65-89).
// Rows past L are zero. Grid (Lpad / 64, H, B), 256 threads. Writes codes to
// codes[(bh * Lpad + row) * D], one scale per block to scales[bh * (Lpad / 64) + blk] and,
// when row_scales != null, the block scale to every row: row_scales[bh * Lpad + row].
template <typename T, int D>
__global__ void __launch_bounds__(256)
block_quant_kernel(const T* __restrict__ x, const float* __restrict__ ksum, int8_t* __restrict__ codes,
                   float* __restrict__ scales, float* __restrict__ row_scales, int L, int H, int Lpad,
                   int64_t sb, int64_t sl, int64_t sh) {
  constexpr int NCH = D / 8;                        // 16-byte chunks per row
  constexpr int PER = kAttnKBlk * NCH / 256;        // chunks per thread (4 or 2)
  const int b = blockIdx.z, h = blockIdx.y, blk = blockIdx.x;
  const int bh = b * H + h;
  const float inv_l = __fdiv_rn(1.0f, static_cast<float>(L));
  float vals[PER][8];
  float amax = 0.f;
#pragma unroll
  for (int u = 0; u < PER; ++u) {
    const int ci = threadIdx.x + u * 256;
    const int r = ci / NCH, c = ci % NCH;
    const int row = blk * kAttnKBlk + r;
    if (row < L) {
      float f[8];
      Vec8<T>::load(x + b * sb + row * sl + h * sh + c * 8, f);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        vals[u][i] = ksum != nullptr ? __fmaf_rn(-ksum[bh * D + c * 8 + i], inv_l, f[i]) : f[i];
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) vals[u][i] = 0.f;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(vals[u][i]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  __shared__ float wmax[8];
  if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = wmax[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) amax = fmaxf(amax, wmax[i]);
  const float inv = amax > 0.f ? __fdiv_rn(127.f, amax) : 0.f;
  const float scale = __fdiv_rn(amax, 127.f);
  if (threadIdx.x == 0 && scales != nullptr) scales[bh * (Lpad / kAttnKBlk) + blk] = scale;
  if (row_scales != nullptr && threadIdx.x < kAttnKBlk)
    row_scales[static_cast<int64_t>(bh) * Lpad + blk * kAttnKBlk + threadIdx.x] = scale;
#pragma unroll
  for (int u = 0; u < PER; ++u) {
    const int ci = threadIdx.x + u * 256;
    const int r = ci / NCH, c = ci % NCH;
    uint32_t w0 = 0, w1 = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      w0 |= code_byte(__fmul_rn(vals[u][i], inv)) << (8 * i);
      w1 |= code_byte(__fmul_rn(vals[u][i + 4], inv)) << (8 * i);
    }
    int8_t* dst = codes + (static_cast<int64_t>(bh) * Lpad + blk * kAttnKBlk + r) * D + c * 8;
    *reinterpret_cast<uint2*>(dst) = make_uint2(w0, w1);
  }
}

// Per-token Q codes (int8_attn_sm80.cu:341-388): amax over the D channels of the row;
// inv = amax > 0 ? 127 / amax : 0; code = rn(x * inv); row scale = amax / 127 (the softmax scale
// is applied by the main kernel). NCH = D / 8 lanes per row; rows in [L, Lpad) are zero.
// Grid (Lpad / (256 / NCH), H, B).
template <typename T, int D>
__global__ void __launch_bounds__(256)
q_token_quant_kernel(const T* __restrict__ q, int8_t* __restrict__ codes, float* __restrict__ row_scales, int L,
                     int H, int Lpad, int64_t sb, int64_t sl, int64_t sh) {
  constexpr int NCH = D / 8;
  constexpr int ROWS_PER_CTA = 256 / NCH;
  const int sub = threadIdx.x / NCH, c = threadIdx.x % NCH;
  const int b = blockIdx.z, h = blockIdx.y;
  const int row = blockIdx.x * ROWS_PER_CTA + sub;
  const int bh = b * H + h;
  const int64_t grow = static_cast<int64_t>(bh) * Lpad + row;
  const bool live = row < Lpad;
  float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (live && row < L) Vec8<T>::load(q + b * sb + row * sl + h * sh + c * 8, f);
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(f[i]));
#pragma unroll
  for (int o = NCH / 2; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float inv = amax > 0.f ? __fdiv_rn(127.f, amax) : 0.f;
  uint32_t w0 = 0, w1 = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    w0 |= code_byte(__fmul_rn(f[i], inv)) << (8 * i);
    w1 |= code_byte(__fmul_rn(f[i + 4], inv)) << (8 * i);
  }
  if (live) {
    *reinterpret_cast<uint2*>(codes + grow * D + c * 8) = make_uint2(w0, w1);
    if (c == 0) row_scales[grow] = __fdiv_rn(amax, 127.f);
  }
}

// ----------------------------------------------------------------------------- main kernel

struct AttnParams {
  int H, Lq, Lk, Lq_pad, Lk_pad, n_ktiles;
  float scale_log2;            // softmax scale * log2(e)
  const float* q_scale;        // [B*H, Lq_pad] per-row Q scale
  const float* k_scale;        // [B*H, Lk_pad / 64] per-block K scale
  void* o;                     // output, (B, Lq, H, D) with the strides below (elements)
  int64_t o_sb, o_sl, o_sh;
  // Key-range split (attn_int8_kernel<..., SPLIT = true> only): CTA x of the grid takes Q pair
  // x / nsplit and key tiles [s tiles_per_split, (s + 1) tiles_per_split) for s = x % nsplit, and
  // writes unnormalized partials for attn_split_combine_kernel instead of O.
  int nsplit = 1, tiles_per_split = 0, BH = 0;
  float* part_o = nullptr;     // [nsplit, B*H, Lq_pad, D] fp32: sum of p v over the range
  float2* part_ml = nullptr;   // [nsplit, B*H, Lq_pad]: (running max m, sum of p) over the range
};

template <int D>
struct AttnSmem {
  static constexpr int kQTile = kAttnBM * D;            // int8
  static constexpr int kKTile = kAttnBN * D;            // int8
  static constexpr int kVTile = kAttnBN * D * 2;        // 16-bit
  static constexpr int kVHalf = kAttnBN * 64 * 2;       // one 64-column TMA box of V
  static constexpr int kStage = kKTile + kVTile;
  static constexpr int kBytes = 2 * kQTile + kAttnStages * kStage;
  static constexpr int kDynamic = kBytes + 1024;
  // Q/K rows are D bytes: 128-byte swizzle for D = 128, 64-byte swizzle for D = 64.
  static constexpr uint32_t kQKSwizzle = D == 128 ? 2u : 4u;   // descriptor layout type
  static constexpr uint32_t kQKAtom = D == 128 ? 1024u : 512u; // 8 rows
};

__device__ __forceinline__ uint64_t smem_desc_sw(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                                 uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  d |= static_cast<uint64_t>(layout & 7u) << 61;
  return d;
}

constexpr int kMagicI = 0x4B400000;         // bits of 1.5 * 2^23
constexpr float kMagicF = 12582912.0f;      // int32 s -> float(s) + 1.5 * 2^23 by an integer add
constexpr float kLazyRescale = 8.0f;        // log2 headroom before O is rescaled

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^a for a pair on the FMA pipe (offloads the MUFU): Cody-Waite style range reduction
// a = j + f, j = rint(a) via the 1.5 * 2^23 rounding constant, f in [-0.5, 0.5]; 2^f by a degree-3
// polynomial fitted here for minimum relative error on [-0.5, 0.5] (max 7.5e-5, far below the
// bf16 / fp16 rounding P receives); 2^j added to the exponent field with an integer add.
// Arguments are clamped at -125 so the exponent field stays positive (2^-125 is 0 for softmax).
__device__ __forceinline__ float2 exp2_poly2(float2 a) {
  a.x = fmaxf(a.x, -125.0f);
  a.y = fmaxf(a.y, -125.0f);
  const float2 magic = make_float2(kMagicF, kMagicF);
  const float2 t = __fadd2_rn(a, magic);                          // j in the low mantissa bits
  const float2 jf = __fadd2_rn(t, make_float2(-kMagicF, -kMagicF));
  const float2 f = __fadd2_rn(a, make_float2(-jf.x, -jf.y));
  float2 p = __ffma2_rn(make_float2(0.0551716685f, 0.0551716685f), f, make_float2(0.2426111400f, 0.2426111400f));
  p = __ffma2_rn(p, f, make_float2(0.6932609677f, 0.6932609677f));
  p = __ffma2_rn(p, f, make_float2(0.9999280572f, 0.9999280572f));
  // bits(t) = bits(1.5 * 2^23) + j and bits(1.5 * 2^23) << 23 == 0 (mod 2^32): (bits(t) << 23) == j << 23
  return make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(t.x) << 23)),
                     __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(t.y) << 23)));
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack_p(float a, float b) {
  if (BF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}


// Max of 64 int32 scores: four independent 3-input-max chains (two new values per op).
__device__ __forceinline__ int row_max64(const uint32_t (&r)[64]) {
  int m4[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    int mx = static_cast<int>(r[16 * c]);
#pragma unroll
    for (int k = 1; k < 15; k += 2)
      mx = __vimax3_s32(mx, static_cast<int>(r[16 * c + k]), static_cast<int>(r[16 * c + k + 1]));
    m4[c] = max(mx, static_cast<int>(r[16 * c + 15]));
  }
  return max(max(m4[0], m4[1]), max(m4[2], m4[3]));
}

__device__ __forceinline__ void mask_tail64(uint32_t (&r)[64], int valid) {
#pragma unroll
  for (int c = 0; c < 64; ++c)
    if (c >= valid) r[c] = static_cast<uint32_t>(INT_MIN);
}

// P for 64 keys of one row: p = 2^(s * c - m) with x = float(s) + 1.5 * 2^23 formed by an integer
// add, so s * c - m = fma(x, c, -(1.5 * 2^23 * c + m)) = fma(x, c, nb), two keys per packed FMA,
// exp2 on the MUFU. Keys at or past `valid` get p = 0 (TAIL only). The sum of p goes to `lsum`
// (four independent accumulators, so no long dependency chain); P as 16-bit pairs to pk[0..31].
// (Measured on a B200: this loop alone, two warps per SM sub-partition, takes 1048 cycles per 64
// keys, MUFU-bound; with a quarter of the exponentials on the FMA pipe (exp2_poly2) 871. In the
// whole kernel at B=1, H=24, L=4608, D=128 that share changed nothing, 253.8 against 252.6 us:
// there one softmax warp alone on its sub-partition takes ~780 cycles per 64 keys, issue- rather
// than MUFU-bound.)
template <bool BF16, bool TAIL>
__device__ __forceinline__ void p_half(const uint32_t (&r)[64], float c, float nb, int valid, float2& lsum,
                                       uint32_t* pk) {
  const float2 cvec = make_float2(c, c), nvec = make_float2(nb, nb);
  float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
  for (int e = 0; e < 32; ++e) {
    const int col = 2 * e;
    const float2 x = make_float2(__int_as_float(static_cast<int>(r[col]) + kMagicI),
                                 __int_as_float(static_cast<int>(r[col + 1]) + kMagicI));
    const float2 a = __ffma2_rn(x, cvec, nvec);
    float2 pr = make_float2(ex2_approx(a.x), ex2_approx(a.y));
    if (TAIL) {
      if (col >= valid) pr.x = 0.f;
      if (col + 1 >= valid) pr.y = 0.f;
    }
    acc[e & 3] = __fadd2_rn(acc[e & 3], pr);
    pk[e] = pack_p<BF16>(pr.x, pr.y);
  }
  lsum = __fadd2_rn(lsum, __fadd2_rn(__fadd2_rn(acc[0], acc[1]), __fadd2_rn(acc[2], acc[3])));
}

__device__ __forceinline__ float scaled_max(int mx, float c) {
  return mx == INT_MIN ? -INFINITY : __fmul_rn(static_cast<float>(mx), c);
}

// SPLIT: this CTA covers one range of key tiles (see AttnParams) and leaves (O, m, l) of it for
// attn_split_combine_kernel; everything inside the range runs as without the split.
template <int D, bool BF16, bool SPLIT = false>
__global__ void __launch_bounds__(kAttnThreads, 1)
attn_int8_kernel(const __grid_constant__ CUtensorMap tma_q, const __grid_constant__ CUtensorMap tma_k,
                 const __grid_constant__ CUtensorMap tma_v, const AttnParams p) {
  using SM = AttnSmem<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sq = smem;                                  // 2 Q tiles
  uint8_t* sstage = smem + 2 * SM::kQTile;             // stages: K tile, then V (D / 64 boxes)

  __shared__ __align__(8) uint64_t q_full;
  __shared__ __align__(8) uint64_t k_full[kAttnStages];
  __shared__ __align__(8) uint64_t v_full[kAttnStages];
  __shared__ __align__(8) uint64_t kv_empty[kAttnStages];
  __shared__ __align__(8) uint64_t s_ready[2];
  __shared__ __align__(8) uint64_t p_ready[2][2];   // [Q tile][key half]
  __shared__ __align__(8) uint64_t pv_done[2][2];
  __shared__ __align__(8) uint64_t drain_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int warp = warp_id(), lane = lane_id();
  const int split = SPLIT ? static_cast<int>(blockIdx.x) % p.nsplit : 0;
  const int qpair = SPLIT ? static_cast<int>(blockIdx.x) / p.nsplit : static_cast<int>(blockIdx.x);
  const int h = blockIdx.y, b = blockIdx.z;
  const int bh = b * p.H + h;
  const int j0 = SPLIT ? split * p.tiles_per_split : 0;               // first key tile of this CTA
  const int n = SPLIT ? min(p.tiles_per_split, p.n_ktiles - j0) : p.n_ktiles;   // key tiles it covers

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    for (int s = 0; s < kAttnStages; ++s) {
      mbar_init(&k_full[s], 1); mbar_init(&v_full[s], 1); mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_ready[i], 1);
      for (int hh = 0; hh < 2; ++hh) { mbar_init(&p_ready[i][hh], 4); mbar_init(&pv_done[i][hh], 1); }
    }
    mbar_init(&drain_bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 8 && lane == 0) { tma_prefetch_desc(&tma_q); tma_prefetch_desc(&tma_k); tma_prefetch_desc(&tma_v); }
  if (warp == 9) { tmem_alloc(&tmem_slot, 512); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  volatile int* abort = &abort_flag;
  // TMEM columns: S0 [0,128), S1 [128,256), O0 [256, 256 + D), O1 [256 + D, 256 + 2D).
  // P_i (16-bit, two keys per column) overwrites S_i half by half: keys 0-63 go to columns
  // [0, 32) once S_i[0, 64) is in registers, keys 64-127 to [64, 96) once S_i[64, 128) is.
  // P.V runs per half, so the tensor core works on one half while the softmax does the other.
  constexpr uint32_t kOCol = 256;

  if (warp == 8) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      bool ok = true;
      const int qrow0 = bh * p.Lq_pad + qpair * kAttnRows;
      mbar_arrive_expect_tx(&q_full, 2 * SM::kQTile);
      tma_load_2d(sq, &tma_q, &q_full, 0, qrow0);
      tma_load_2d(sq + SM::kQTile, &tma_q, &q_full, 0, qrow0 + kAttnBM);
      for (int j = 0; j < n && ok; ++j) {
        const int st = j % kAttnStages;
        const uint32_t ph = (j / kAttnStages) & 1;
        if (!mbar_wait(&kv_empty[st], ph ^ 1, abort)) { ok = false; break; }
        uint8_t* sk = sstage + st * SM::kStage;
        uint8_t* sv = sk + SM::kKTile;
        mbar_arrive_expect_tx(&k_full[st], SM::kKTile);
        tma_load_2d(sk, &tma_k, &k_full[st], 0, bh * p.Lk_pad + (j0 + j) * kAttnBN);
        mbar_arrive_expect_tx(&v_full[st], SM::kVTile);
#pragma unroll
        for (int dh = 0; dh < D / 64; ++dh)
          tma_load_4d(sv + dh * SM::kVHalf, &tma_v, &v_full[st], dh * 64, (j0 + j) * kAttnBN, h, b);
      }
      if (!ok) for (int i = 0; i < 1000; ++i) __nanosleep(1000);
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------------ MMA issuer (lane 0)
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_i8(kAttnBM, kAttnBN);
      constexpr uint32_t idesc_o = idesc_f16(kAttnBM, D, BF16, true);
      const uint32_t sq_addr = smem_u32(sq);
      // Descriptors advance by adding to the start-address field (bits 0-13, in 16-byte units).
      auto issue_s = [&](int i, int st) {
        const uint32_t sk_addr = smem_u32(sstage + st * SM::kStage);
        uint64_t ad = smem_desc_sw(sq_addr + i * SM::kQTile, 16, SM::kQKAtom, SM::kQKSwizzle);
        uint64_t bd = smem_desc_sw(sk_addr, 16, SM::kQKAtom, SM::kQKSwizzle);
        const uint32_t d = tmem + i * 128;
#pragma unroll
        for (int kk = 0; kk < D / 32; ++kk) {
          mma_i8_ss(d, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
          ad += 32 >> 4;
          bd += 32 >> 4;
        }
      };
      // O_i += P_i[:, 64 keys of half hh] . V[those keys, :]. B = V rows, MN-major, 128B swizzle:
      // 8-key groups 1024 B apart, 64-column boxes kVHalf apart; each step moves 16 keys (2048 B).
      auto issue_pv = [&](int i, int hh, int st, bool acc) {
        uint64_t bd = smem_desc_sw(smem_u32(sstage + st * SM::kStage + SM::kKTile) + hh * 64 * 128, SM::kVHalf,
                                   1024, 2);
        const uint32_t d = tmem + kOCol + i * D;
        uint32_t a = tmem + i * 128 + hh * 64;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          mma_f16_ts(d, a, bd, idesc_o, (acc || kk > 0) ? 1u : 0u);
          bd += 2048 >> 4;
          a += 8;
        }
      };
      bool ok = mbar_wait(&q_full, 0, abort) && mbar_wait(&k_full[0], 0, abort);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0); mma_commit(&s_ready[0]);
        issue_s(1, 0); mma_commit(&s_ready[1]);
      }
      // In the loop, descriptors are stage 0's plus st * kStage in the start-address field, both
      // waits on the stages (this tile's V, the next tile's K, loaded stages ahead) come first, and the
      // MMA thread then only waits on P between its MMA groups.
      const uint64_t qd0 = smem_desc_sw(sq_addr, 16, SM::kQKAtom, SM::kQKSwizzle);
      const uint64_t kd0 = smem_desc_sw(smem_u32(sstage), 16, SM::kQKAtom, SM::kQKSwizzle);
      const uint64_t vd0 = smem_desc_sw(smem_u32(sstage + SM::kKTile), SM::kVHalf, 1024, 2);
      for (int j = 0; j < n && ok; ++j) {
        const int st = j % kAttnStages;
        const uint32_t ph = (j / kAttnStages) & 1;
        const int st1 = (j + 1) % kAttnStages;
        const uint32_t ph1 = ((j + 1) / kAttnStages) & 1;
        const bool more = j + 1 < n;
        if (!mbar_wait(&v_full[st], ph, abort)) { ok = false; break; }
        if (more && !mbar_wait(&k_full[st1], ph1, abort)) { ok = false; break; }
        const uint64_t vd = vd0 + static_cast<uint64_t>(st * (SM::kStage >> 4));
        const uint64_t kd = kd0 + static_cast<uint64_t>(st1 * (SM::kStage >> 4));
#pragma unroll
        for (int i = 0; i < 2; ++i) {
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            if (ok) ok = mbar_wait(&p_ready[i][hh], j & 1, abort);
            if (ok) {
              tc_fence_after();
              // O_i += P_i[:, 64 keys of half hh] . V[those keys, :] (see issue_pv)
              uint64_t bd = vd + static_cast<uint64_t>((hh * 64 * 128) >> 4);
              const uint32_t d = tmem + kOCol + i * D;
              uint32_t a = tmem + i * 128 + hh * 64;
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) {
                mma_f16_ts(d, a, bd, idesc_o, (j > 0 || hh > 0 || kk > 0) ? 1u : 0u);
                bd += 2048 >> 4;
                a += 8;
              }
              mma_commit(&pv_done[i][hh]);
            }
          }
          if (ok && i == 1) mma_commit(&kv_empty[st]);
          if (ok && more) {
            uint64_t ad = qd0 + static_cast<uint64_t>((i * SM::kQTile) >> 4);
            uint64_t bd = kd;
            const uint32_t d = tmem + i * 128;
#pragma unroll
            for (int kk = 0; kk < D / 32; ++kk) {
              mma_i8_ss(d, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
              ad += 32 >> 4;
              bd += 32 >> 4;
            }
            mma_commit(&s_ready[i]);
          }
        }
      }
      mma_commit(&drain_bar);
      mbar_wait(&drain_bar, 0, nullptr, 1000000);
    }
  } else {
    // ------------------------------------------------------------------ softmax warpgroups
    const int wg = warp >> 2;                 // Q tile 0 or 1
    const int quarter = warp & 3;             // TMEM lane quarter
    const int r_local = quarter * 32 + lane;
    const int qrow = qpair * kAttnRows + wg * kAttnBM + r_local;    // row in [0, Lq_pad)
    const float cq = __fmul_rn(p.q_scale[static_cast<int64_t>(bh) * p.Lq_pad + qrow], p.scale_log2);
    // K scales from this CTA's first key tile on (two 64-key blocks per tile)
    const float* ksc = p.k_scale + static_cast<int64_t>(bh) * (p.Lk_pad / kAttnKBlk) + 2 * j0;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_addr = tmem + lane_off + wg * 128;
    const uint32_t o_addr = tmem + lane_off + kOCol + wg * D;
    const int tail_valid = p.Lk - (p.n_ktiles - 1) * kAttnBN;      // keys in the last tile (1..128)
    const bool last_range = j0 + n == p.n_ktiles;                   // this CTA holds that tile
    float m = -INFINITY;
    float2 l2 = make_float2(0.f, 0.f);
    float ks_cur[2] = {ksc[0], ksc[1]};
    bool ok = true;
    // Multiply this row of O by alpha once every P.V issued so far for this Q tile has landed
    // (waiting for `bar` at `parity`, the latest of them). Rare: only when the running max moves.
    auto rescale_o = [&](uint64_t* bar, uint32_t parity, float alpha) -> bool {
      bool w = mbar_wait(bar, parity, abort);
      if (!__all_sync(0xffffffffu, w)) return false;
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < D; c += 32) {
        uint32_t o[32];
        tmem_ld32(o_addr + c, o);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const float2 v = __fmul2_rn(make_float2(__uint_as_float(o[e]), __uint_as_float(o[e + 1])),
                                      make_float2(alpha, alpha));
          o[e] = __float_as_uint(v.x);
          o[e + 1] = __float_as_uint(v.y);
        }
        tmem_st32(o_addr + c, o);
      }
      return true;
    };
    uint32_t r[64];
    for (int j = 0; j < n && ok; ++j) {
      // next tile's K scales, loaded a tile ahead so their latency hides behind this one
      float ks_next[2] = {0.f, 0.f};
      if (j + 1 < n) { ks_next[0] = ksc[2 * j + 2]; ks_next[1] = ksc[2 * j + 3]; }
      ok = mbar_wait(&s_ready[wg], j & 1, abort);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      tc_fence_after();
      const bool tail = j == n - 1 && last_range && tail_valid < kAttnBN;
      tmem_ld32(s_addr + 0, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
      tmem_ld32(s_addr + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
      tmem_wait_ld();
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        // r holds S[:, 64 hh, 64 hh + 64) here.
        const int valid = tail ? tail_valid - 64 * hh : 64;
        if (valid < 64) mask_tail64(r, valid);
        const float c = __fmul_rn(cq, ks_cur[hh]);
        const int mx = row_max64(r);
        if (j == 0 && hh == 0) m = scaled_max(mx, c);    // the running max starts at tile 0's first half
        // P with the running max; if this half's max exceeds it by more than 2^8 somewhere in the
        // warp, move the max up, recompute from the registers in hand and rescale O.
        float2 lt = make_float2(0.f, 0.f);
        uint32_t pk[32];
        if (valid < 64) p_half<BF16, true>(r, c, -__fmaf_rn(kMagicF, c, m), valid, lt, pk);
        else p_half<BF16, false>(r, c, -__fmaf_rn(kMagicF, c, m), valid, lt, pk);
        const float mt = scaled_max(mx, c);
        if (__any_sync(0xffffffffu, mt > m + kLazyRescale)) {
          const float mnew = fmaxf(m, mt);
          const float alpha = ex2_approx(m - mnew);
          l2 = __fmul2_rn(l2, make_float2(alpha, alpha));
          m = mnew;
          lt = make_float2(0.f, 0.f);
          if (valid < 64) p_half<BF16, true>(r, c, -__fmaf_rn(kMagicF, c, m), valid, lt, pk);
          else p_half<BF16, false>(r, c, -__fmaf_rn(kMagicF, c, m), valid, lt, pk);
          // O holds P.V of every half before this one: tile j-1's second half, or tile j's first.
          const bool have_o = j > 0 || hh > 0;
          if (have_o) {
            const bool w = hh == 0 ? rescale_o(&pv_done[wg][1], (j - 1) & 1, alpha)
                                   : rescale_o(&pv_done[wg][0], j & 1, alpha);
            if (!w) { ok = false; break; }
          }
        }
        l2 = __fadd2_rn(l2, lt);
        if (hh == 0) {
          // prefetch the second half while P of the first is stored
          tmem_ld32(s_addr + 64, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
          tmem_ld32(s_addr + 96, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
        }
        tmem_st32(s_addr + 64 * hh, pk);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_ready[wg][hh]);
        if (hh == 0) tmem_wait_ld();
      }
      ks_cur[0] = ks_next[0];
      ks_cur[1] = ks_next[1];
    }
    if (ok) {
      ok = mbar_wait(&pv_done[wg][1], (n - 1) & 1, abort);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (SPLIT && ok) {
      // this key range's unnormalized O, running max and sum, for attn_split_combine_kernel
      tc_fence_after();
      const bool row_ok = qrow < p.Lq;
      const int64_t prow = (static_cast<int64_t>(split) * p.BH + bh) * p.Lq_pad + qrow;
      float* dst = p.part_o + prow * D;
#pragma unroll 1
      for (int c = 0; c < D; c += 32) {
        uint32_t o[32];
        tmem_ld32(o_addr + c, o);
        tmem_wait_ld();
        if (row_ok) {
#pragma unroll
          for (int e = 0; e < 32; e += 4)
            *reinterpret_cast<uint4*>(dst + c + e) = make_uint4(o[e], o[e + 1], o[e + 2], o[e + 3]);
        }
      }
      if (row_ok) p.part_ml[prow] = make_float2(m, __fadd_rn(l2.x, l2.y));
    } else if (ok) {
      tc_fence_after();
      const float inv = __fdiv_rn(1.0f, __fadd_rn(l2.x, l2.y));
      const bool row_ok = qrow < p.Lq;
      uint16_t* dst = reinterpret_cast<uint16_t*>(p.o) + b * p.o_sb + static_cast<int64_t>(qrow) * p.o_sl + h * p.o_sh;
#pragma unroll 1
      for (int c = 0; c < D; c += 32) {
        uint32_t o[32];
        tmem_ld32(o_addr + c, o);
        tmem_wait_ld();
        if (row_ok) {
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            uint4 w;
            w.x = pack_p<BF16>(__fmul_rn(__uint_as_float(o[e]), inv), __fmul_rn(__uint_as_float(o[e + 1]), inv));
            w.y = pack_p<BF16>(__fmul_rn(__uint_as_float(o[e + 2]), inv), __fmul_rn(__uint_as_float(o[e + 3]), inv));
            w.z = pack_p<BF16>(__fmul_rn(__uint_as_float(o[e + 4]), inv), __fmul_rn(__uint_as_float(o[e + 5]), inv));
            w.w = pack_p<BF16>(__fmul_rn(__uint_as_float(o[e + 6]), inv), __fmul_rn(__uint_as_float(o[e + 7]), inv));
            *reinterpret_cast<uint4*>(dst + c + e) = w;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ----------------------------------------------------------------------------- split combine
// One warp per query row: the key ranges' partials (O_s, m_s, l_s) of attn_int8_kernel<..., SPLIT>
// merged as o = sum_s 2^(m_s - M) O_s / sum_s 2^(m_s - M) l_s with M = max_s m_s (p was
// 2^(s c - m_s) in range s), in split order, rounded once to the output dtype. D / 32 consecutive
// columns per lane.
template <int D, bool BF16>
__global__ void __launch_bounds__(256)
attn_split_combine_kernel(const float* __restrict__ part_o, const float2* __restrict__ part_ml, int nsplit, int BH,
                          int H, int Lq, int Lq_pad, void* __restrict__ o, int64_t o_sb, int64_t o_sl, int64_t o_sh) {
  constexpr int kPer = D / 32;
  const int64_t wrow = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wrow >= static_cast<int64_t>(BH) * Lq) return;
  const int bh = static_cast<int>(wrow / Lq), row = static_cast<int>(wrow % Lq);
  const int64_t split_stride = static_cast<int64_t>(BH) * Lq_pad;      // partial rows per split
  const int64_t base = static_cast<int64_t>(bh) * Lq_pad + row;
  float mmax = -INFINITY;
  for (int sp = 0; sp < nsplit; ++sp) mmax = fmaxf(mmax, part_ml[sp * split_stride + base].x);
  float acc[kPer];
#pragma unroll
  for (int e = 0; e < kPer; ++e) acc[e] = 0.f;
  float den = 0.f;
  for (int sp = 0; sp < nsplit; ++sp) {
    const float2 ml = part_ml[sp * split_stride + base];
    const float w = exp2f(ml.x - mmax);
    den = __fmaf_rn(w, ml.y, den);
    const float* src = part_o + (sp * split_stride + base) * D + lane * kPer;
    float v[kPer];
    if constexpr (kPer == 4) {
      const float4 t = *reinterpret_cast<const float4*>(src);
      v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
    } else {
      const float2 t = *reinterpret_cast<const float2*>(src);
      v[0] = t.x; v[1] = t.y;
    }
#pragma unroll
    for (int e = 0; e < kPer; ++e) acc[e] = __fmaf_rn(w, v[e], acc[e]);
  }
  const float inv = __fdiv_rn(1.0f, den);
  const int b = bh / H, h = bh % H;
  uint16_t* dst = reinterpret_cast<uint16_t*>(o) + b * o_sb + static_cast<int64_t>(row) * o_sl + h * o_sh + lane * kPer;
  if constexpr (kPer == 4) {
    *reinterpret_cast<uint2*>(dst) = make_uint2(pack_p<BF16>(__fmul_rn(acc[0], inv), __fmul_rn(acc[1], inv)),
                                                pack_p<BF16>(__fmul_rn(acc[2], inv), __fmul_rn(acc[3], inv)));
  } else {
    *reinterpret_cast<uint32_t*>(dst) = pack_p<BF16>(__fmul_rn(acc[0], inv), __fmul_rn(acc[1], inv));
  }
}

// ----------------------------------------------------------------------------- main kernel, S double-buffered
//
// One CTA per 128-row Q tile. TMEM holds two S buffers and O: S(j) lands in buffer j & 1 while
// the softmax works on S(j - 1) from the other, so Q.K^T of the next tile runs on the tensor core
// during the exponentials of this one. P(j) is written over the S(j) columns its warp has already
// read, so the buffer is free again once P.V(j) has run (the MMA that overwrites it with S(j + 2)
// is issued after P.V(j), and tcgen05 MMAs of one CTA execute in issue order).
//   warps 0-7   softmax: warp w owns TMEM lane quarter w & 3 (32 query rows) and key half w >> 2
//               (64 of the tile's 128 keys): two warps per row, two per SM sub-partition
//   warp 8      TMA producer (Q once; K and V per stage)
//   warp 9      TMEM allocator + MMA issuer
// The two warps of a row exchange their half-row maxima once per tile through shared memory
// (a bounded mbarrier round), so both apply the same running max; their partial row sums are
// added at the end. O is rescaled lazily (only when the row max grows by more than 2^8), each warp
// its half of the columns.
constexpr int kDbRows = 128;
constexpr int kDbStages = 3;

template <int D>
struct AttnDbSmem {
  static constexpr int kQTile = kDbRows * D;
  static constexpr int kKTile = kAttnBN * D;
  static constexpr int kVTile = kAttnBN * D * 2;
  static constexpr int kVHalf = kAttnBN * 64 * 2;
  static constexpr int kStage = kKTile + kVTile;
  static constexpr int kBytes = kQTile + kDbStages * kStage;
  static constexpr int kDynamic = kBytes + 1024;
  static constexpr uint32_t kQKSwizzle = D == 128 ? 2u : 4u;
  static constexpr uint32_t kQKAtom = D == 128 ? 1024u : 512u;
};

template <int D, bool BF16>
__global__ void __launch_bounds__(kAttnThreads, 1)
attn_db_kernel(const __grid_constant__ CUtensorMap tma_q, const __grid_constant__ CUtensorMap tma_k,
               const __grid_constant__ CUtensorMap tma_v, const AttnParams p) {
  using SM = AttnDbSmem<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sq = smem;
  uint8_t* sstage = smem + SM::kQTile;

  __shared__ __align__(8) uint64_t q_full;
  __shared__ __align__(8) uint64_t k_full[kDbStages];
  __shared__ __align__(8) uint64_t v_full[kDbStages];
  __shared__ __align__(8) uint64_t kv_empty[kDbStages];
  __shared__ __align__(8) uint64_t s_full[2];
  __shared__ __align__(8) uint64_t p_full[2];
  __shared__ __align__(8) uint64_t pv_done;
  __shared__ __align__(8) uint64_t pair_bar[4];      // per lane quarter: the two warps of those rows
  __shared__ __align__(8) uint64_t drain_bar;
  __shared__ float s_xchg[2][2][kDbRows];             // [tile parity][key half][row]
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int warp = warp_id(), lane = lane_id();
  const int qtile = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int bh = b * p.H + h;
  const int n = p.n_ktiles;

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    for (int s = 0; s < kDbStages; ++s) { mbar_init(&k_full[s], 1); mbar_init(&v_full[s], 1); mbar_init(&kv_empty[s], 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(&s_full[i], 1); mbar_init(&p_full[i], 8); }
    mbar_init(&pv_done, 1);
    for (int i = 0; i < 4; ++i) mbar_init(&pair_bar[i], 64);
    mbar_init(&drain_bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 8 && lane == 0) { tma_prefetch_desc(&tma_q); tma_prefetch_desc(&tma_k); tma_prefetch_desc(&tma_v); }
  if (warp == 9) { tmem_alloc(&tmem_slot, 512); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  volatile int* abort = &abort_flag;
  constexpr uint32_t kOCol = 256;   // S buffers at [0, 128) and [128, 256), O at [256, 256 + D)

  if (warp == 8) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      bool ok = true;
      mbar_arrive_expect_tx(&q_full, SM::kQTile);
      tma_load_2d(sq, &tma_q, &q_full, 0, bh * p.Lq_pad + qtile * kDbRows);
      for (int j = 0; j < n && ok; ++j) {
        const int st = j % kDbStages;
        const uint32_t ph = (j / kDbStages) & 1;
        if (!mbar_wait(&kv_empty[st], ph ^ 1, abort)) { ok = false; break; }
        uint8_t* sk = sstage + st * SM::kStage;
        uint8_t* sv = sk + SM::kKTile;
        mbar_arrive_expect_tx(&k_full[st], SM::kKTile);
        tma_load_2d(sk, &tma_k, &k_full[st], 0, bh * p.Lk_pad + j * kAttnBN);
        mbar_arrive_expect_tx(&v_full[st], SM::kVTile);
#pragma unroll
        for (int dh = 0; dh < D / 64; ++dh)
          tma_load_4d(sv + dh * SM::kVHalf, &tma_v, &v_full[st], dh * 64, j * kAttnBN, h, b);
      }
      if (!ok) for (int i = 0; i < 1000; ++i) __nanosleep(1000);
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------------ MMA issuer (lane 0)
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_i8(kDbRows, kAttnBN);
      constexpr uint32_t idesc_o = idesc_f16(kDbRows, D, BF16, true);
      const uint32_t sq_addr = smem_u32(sq);
      auto issue_s = [&](int buf, int st) {
        uint64_t ad = smem_desc_sw(sq_addr, 16, SM::kQKAtom, SM::kQKSwizzle);
        uint64_t bd = smem_desc_sw(smem_u32(sstage + st * SM::kStage), 16, SM::kQKAtom, SM::kQKSwizzle);
        const uint32_t d = tmem + buf * 128;
#pragma unroll
        for (int kk = 0; kk < D / 32; ++kk) {
          mma_i8_ss(d, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
          ad += 32 >> 4;
          bd += 32 >> 4;
        }
      };
      // O += P(buf) . V(stage): 16 keys per MMA; P of keys [64 hf, 64 hf + 64) sits at columns
      // [64 hf, 64 hf + 32) of the buffer (two keys per column).
      auto issue_pv = [&](int buf, int st, bool acc) {
        const uint64_t bd0 = smem_desc_sw(smem_u32(sstage + st * SM::kStage + SM::kKTile), SM::kVHalf, 1024, 2);
        const uint32_t d = tmem + kOCol;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t a = tmem + buf * 128 + (kk >> 2) * 64 + (kk & 3) * 8;
          mma_f16_ts(d, a, bd0 + static_cast<uint64_t>((kk * 2048) >> 4), idesc_o, (acc || kk > 0) ? 1u : 0u);
        }
      };
      bool ok = mbar_wait(&q_full, 0, abort) && mbar_wait(&k_full[0], 0, abort);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        mma_commit(&s_full[0]);
      }
      if (ok && n > 1) {
        ok = mbar_wait(&k_full[1 % kDbStages], (1 / kDbStages) & 1, abort);
        if (ok) {
          tc_fence_after();
          issue_s(1, 1 % kDbStages);
          mma_commit(&s_full[1]);
        }
      }
      for (int j = 0; j < n && ok; ++j) {
        const int buf = j & 1;
        const int st = j % kDbStages;
        if (!mbar_wait(&p_full[buf], (j >> 1) & 1, abort)) { ok = false; break; }
        if (!mbar_wait(&v_full[st], (j / kDbStages) & 1, abort)) { ok = false; break; }
        tc_fence_after();
        issue_pv(buf, st, j > 0);
        mma_commit(&pv_done);
        mma_commit(&kv_empty[st]);
        if (j + 2 < n) {
          const int st2 = (j + 2) % kDbStages;
          if (!mbar_wait(&k_full[st2], ((j + 2) / kDbStages) & 1, abort)) { ok = false; break; }
          tc_fence_after();
          issue_s(buf, st2);
          mma_commit(&s_full[buf]);
        }
      }
      mma_commit(&drain_bar);
      mbar_wait(&drain_bar, 0, nullptr, 1000000);
    }
  } else {
    // ------------------------------------------------------------------ softmax warps
    const int quarter = warp & 3;
    const int hf = warp >> 2;                 // key half of every tile this warp owns
    const int r_local = quarter * 32 + lane;
    const int qrow = qtile * kDbRows + r_local;
    const float cq = __fmul_rn(p.q_scale[static_cast<int64_t>(bh) * p.Lq_pad + qrow], p.scale_log2);
    const float* ksc = p.k_scale + static_cast<int64_t>(bh) * (p.Lk_pad / kAttnKBlk);
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    constexpr int kOHalf = D / 2;             // O columns this warp rescales and stores
    const uint32_t o_addr = tmem + lane_off + kOCol + hf * kOHalf;
    const int tail_valid = p.Lk - (n - 1) * kAttnBN;
    float m = -INFINITY;
    float2 l2 = make_float2(0.f, 0.f);
    float ks_cur = ksc[hf];
    bool ok = true;
    uint32_t r[64];
    // both warps of these rows meet here; returns false if the round did not complete
    auto pair_round = [&](int round) -> bool {
      mbar_arrive(&pair_bar[quarter]);
      return mbar_wait(&pair_bar[quarter], round & 1, abort);
    };
    for (int j = 0; j < n && ok; ++j) {
      const int buf = j & 1;
      const float ks_next = j + 1 < n ? ksc[2 * (j + 1) + hf] : 0.f;
      ok = mbar_wait(&s_full[buf], (j >> 1) & 1, abort);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      tc_fence_after();
      const uint32_t s_addr = tmem + lane_off + buf * 128 + hf * 64;
      tmem_ld32(s_addr, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
      tmem_ld32(s_addr + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
      tmem_wait_ld();
      const int valid = (j == n - 1) ? tail_valid - 64 * hf : 64;
      if (valid < 64) mask_tail64(r, valid);
      const float c = __fmul_rn(cq, ks_cur);
      const float mt = scaled_max(row_max64(r), c);
      s_xchg[j & 1][hf][r_local] = mt;
      ok = pair_round(j);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      const float row_mt = fmaxf(mt, s_xchg[j & 1][hf ^ 1][r_local]);
      if (j == 0) {
        m = row_mt;
      } else if (__any_sync(0xffffffffu, row_mt > m + kLazyRescale)) {
        // Rare: move the running max up and rescale this warp's half of O once P.V(j - 1) landed.
        // The branch is warp-uniform (its body holds warp-collective tcgen05 loads/stores); rows
        // whose max did not move get alpha = 1. Both warps of these rows see the same row maxima,
        // so they take the branch together.
        const float mnew = fmaxf(m, row_mt);
        const float alpha = ex2_approx(m - mnew);
        l2 = __fmul2_rn(l2, make_float2(alpha, alpha));
        m = mnew;
        ok = mbar_wait(&pv_done, (j - 1) & 1, abort);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        tc_fence_after();
#pragma unroll 1
        for (int cc = 0; cc < kOHalf; cc += 32) {
          uint32_t o[32];
          tmem_ld32(o_addr + cc, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            const float2 v = __fmul2_rn(make_float2(__uint_as_float(o[e]), __uint_as_float(o[e + 1])),
                                        make_float2(alpha, alpha));
            o[e] = __float_as_uint(v.x);
            o[e + 1] = __float_as_uint(v.y);
          }
          tmem_st32(o_addr + cc, o);
        }
      }
      float2 lt = make_float2(0.f, 0.f);
      uint32_t pk[32];
      if (valid < 64) p_half<BF16, true>(r, c, -__fmaf_rn(kMagicF, c, m), valid, lt, pk);
      else p_half<BF16, false>(r, c, -__fmaf_rn(kMagicF, c, m), valid, lt, pk);
      l2 = __fadd2_rn(l2, lt);
      tmem_st32(tmem + lane_off + buf * 128 + hf * 64, pk);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[buf]);
      ks_cur = ks_next;
    }
    if (ok) {
      ok = mbar_wait(&pv_done, (n - 1) & 1, abort);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok) {
      s_xchg[n & 1][hf][r_local] = __fadd_rn(l2.x, l2.y);
      ok = pair_round(n);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok) {
      tc_fence_after();
      const float l_row = __fadd_rn(s_xchg[n & 1][0][r_local], s_xchg[n & 1][1][r_local]);
      const float inv = __fdiv_rn(1.0f, l_row);
      const bool row_ok = qrow < p.Lq;
      uint16_t* dst = reinterpret_cast<uint16_t*>(p.o) + b * p.o_sb + static_cast<int64_t>(qrow) * p.o_sl + h * p.o_sh +
                      hf * kOHalf;
#pragma unroll 1
      for (int cc = 0; cc < kOHalf; cc += 32) {
        uint32_t o[32];
        tmem_ld32(o_addr + cc, o);
        tmem_wait_ld();
        if (row_ok) {
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            uint4 w;
            w.x = pack_p<BF16>(__fmul_rn(__uint_as_float(o[e]), inv), __fmul_rn(__uint_as_float(o[e + 1]), inv));
            w.y = pack_p<BF16>(__fmul_rn(__uint_as_float(o[e + 2]), inv), __fmul_rn(__uint_as_float(o[e + 3]), inv));
            w.z = pack_p<BF16>(__fmul_rn(__uint_as_float(o[e + 4]), inv), __fmul_rn(__uint_as_float(o[e + 5]), inv));
            w.w = pack_p<BF16>(__fmul_rn(__uint_as_float(o[e + 6]), inv), __fmul_rn(__uint_as_float(o[e + 7]), inv));
            *reinterpret_cast<uint4*>(dst + cc + e) = w;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace dc
