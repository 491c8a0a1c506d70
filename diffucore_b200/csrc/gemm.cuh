// W8A8 GEMM on the sm_100a tensor core: out[M, N] = epilogue(q[M, K] . w[N, K]^T).
//
// Persistent, warp-specialised kernel, one CTA per SM:
//   warp 0      TMA producer: A (activations) and B (weights) tiles, 128-byte swizzle
//   warp 1      TMEM allocator + single-thread tcgen05.mma.kind::i8 issuer
//   warps 2..5  epilogue: tcgen05.ld of the int32 accumulator, rescale, bias, store
// Accumulators live in TMEM, double-buffered (2 x BN columns) so the epilogue of one tile
// overlaps the main loop of the next.
//
// PAIR runs the same roles in a cluster of two CTAs on one TPC with 256 x BN tiles: each CTA
// stages its 128 rows of A and half (BN/2 rows) of B per k-block, the even CTA's MMA thread issues
// `cta_group::2` MMAs that read both CTAs' shared memory and write each CTA's 128 accumulator rows
// into that CTA's TMEM, and each CTA's epilogue drains its own rows. Per SM that halves the B bytes
// TMA writes and the tensor core reads per k-block (32 KB instead of 48 KB per 128 x 256 x 128),
// the shared-memory traffic that limits the one-CTA tile. Barriers: both CTAs' loads of a stage
// count on the even CTA's `full_bar`; its MMA commits arrive on both CTAs' `empty_bar` and
// `acc_full` (one commit with CTA mask 0b11); both CTAs' epilogue warps arrive on the even CTA's
// `acc_empty`.
//
// The epilogue rounds exactly like the reference's `rescale` (src/diffucore/models/_int8.py:313-323):
//   y = dtype(float(acc) * (sx[m] * sw[n]));  if bias: y = dtype(float(y) + float(bias[n]))
// and with OUT_I32 it writes the raw accumulator (the reference's `int_mm`, _int8.py:200-207).
// GATED adds a DiT residual branch in the same pass: out = dtype(res + dtype(gate[n] * y)), the
// rounding of `x + mod.gate * linear(h)` in the model dtype (src/diffucore/models/flux_dit.py:302-305,
// :339); res may be the output itself (each element is read before it is written, by one thread).
// A column-block output (col_block > 0) stores column n of row m at
//   out + (n / col_block) * block_stride + m * ldo + n % col_block,
// which lays a projection's output out as [blocks, M, col_block] for an all-to-all.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>
#include "sm100.cuh"

namespace dc {

enum GemmOut : int { kOutBF16 = 0, kOutF16 = 1, kOutI32 = 2 };

constexpr int kGemmBM = 128;
constexpr int kGemmAtom = 128;          // bytes = int8 elements of K per 128B swizzle row (one TMA box)
constexpr int kGemmEpiWarps = 8;        // two warps per TMEM lane quarter, each half of the columns
constexpr int kGemmThreads = 64 + 32 * kGemmEpiWarps;

struct GemmParams {
  int M, N, K;
  int tiles_m, tiles_n, num_tiles, num_kb;
  const float* sx;
  const float* sw;
  const void* bias;      // dtype of the output (bf16 / fp16), or null
  void* out;
  int64_t ldo;           // output row stride in elements
  const void* gate;      // GATED: [N] in the output dtype
  const void* residual;  // GATED: [M, N] with row stride ldr, in the output dtype
  int64_t ldr;
  int64_t col_block;     // 0: plain [M, N] output; else a multiple of BN (see above)
  int64_t block_stride;  // elements between column blocks
  int out_vec;           // 16-byte stores allowed: out 16-byte aligned, ldo and block_stride rows of 16 B
  int res_vec;           // 16-byte residual loads allowed: residual 16-byte aligned, ldr rows of 16 B
};

// A k-block is KATOMS swizzle atoms of 128 bytes of K: A then B, each atom [rows][128 B].
template <int BN, int STAGES, int KATOMS>
struct GemmSmem {
  static constexpr int kBK = KATOMS * kGemmAtom;    // int8 elements of K per k-block
  static constexpr int kAtomA = kGemmBM * kGemmAtom;
  static constexpr int kAtomB = BN * kGemmAtom;
  static constexpr int kA = KATOMS * kAtomA;
  static constexpr int kB = KATOMS * kAtomB;
  static constexpr int kStage = kA + kB;
  static constexpr int kBytes = STAGES * kStage;
  static constexpr int kDynamic = kBytes + 1024;    // slack for 1024-byte alignment
};

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack_f16x2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

template <int OUT>
__device__ __forceinline__ float out_round(float y) {
  if (OUT == kOutBF16) return __bfloat162float(__float2bfloat16_rn(y));
  return __half2float(__float2half_rn(y));
}

template <int OUT>
__device__ __forceinline__ float bias_at(const void* bias, int n) {
  if (OUT == kOutBF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(bias)[n]);
  return __half2float(reinterpret_cast<const __half*>(bias)[n]);
}

// y = dtype(float(acc) * (sx * sw)); y = dtype(float(y) + bias); y = GELU(y) in dtype. The value
// returned is exactly representable in the output dtype, so the final pack does not round again.
template <int OUT, bool HAS_BIAS, int GELU>
__device__ __forceinline__ float epi_value(uint32_t acc_bits, float sxr, float swn, float bn) {
  const float a = __int2float_rn(static_cast<int>(acc_bits));
  float y = out_round<OUT>(__fmul_rn(a, __fmul_rn(sxr, swn)));
  if (HAS_BIAS) y = out_round<OUT>(__fadd_rn(y, bn));
  if (GELU != 0) {
    if (OUT == kOutBF16) y = gelu_dtype<__nv_bfloat16>(y, GELU);
    else y = gelu_dtype<__half>(y, GELU);
  }
  return y;
}

// out = dtype(res + dtype(gate * y)), res given as its 16-bit pattern.
template <int OUT>
__device__ __forceinline__ float gated_residual(uint32_t res_bits, float gate, float y) {
  const float rv = OUT == kOutBF16 ? __uint_as_float(res_bits << 16)
                                   : __half2float(__ushort_as_half(static_cast<unsigned short>(res_bits)));
  return out_round<OUT>(__fadd_rn(rv, out_round<OUT>(__fmul_rn(gate, y))));
}

// KATOMS: 128-byte atoms of K per pipeline stage. Two (256-byte k-blocks) halve the barrier round
// trips between the TMA producer and the MMA thread per byte of K.
template <int BN, int STAGES, int OUT, bool HAS_BIAS, int GELU, bool GATED = false, bool PAIR = false,
          int KATOMS = 1>
__global__ void __launch_bounds__(kGemmThreads, 1)
gemm_w8a8_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                 const GemmParams p) {
  using S = GemmSmem<PAIR ? BN / 2 : BN, STAGES, KATOMS>;  // B rows staged by this CTA
  constexpr int kHalf = BN / 2;                 // columns per epilogue warp
  constexpr int kTileM = PAIR ? 2 * kGemmBM : kGemmBM;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ __align__(8) uint64_t empty_bar[STAGES];
  __shared__ __align__(8) uint64_t acc_full[2];
  __shared__ __align__(8) uint64_t acc_empty[2];
  __shared__ __align__(8) uint64_t drain_bar;
  __shared__ __align__(16) float col_sw[kGemmEpiWarps][kHalf];    // per-warp staging of sw / bias
  __shared__ __align__(16) float col_bias[kGemmEpiWarps][kHalf];
  __shared__ __align__(16) float col_gate[GATED ? kGemmEpiWarps : 1][GATED ? kHalf : 4];
  // per epilogue warp: one 32-row x 32-column 16-bit block, 16-byte units swizzled (epi_unit)
  __shared__ __align__(16) uint4 epi_tile[OUT == kOutI32 ? 1 : kGemmEpiWarps][OUT == kOutI32 ? 1 : 128];
  __shared__ uint32_t tmem_base_slot;
  __shared__ int abort_flag;

  const int warp = warp_id(), lane = lane_id();
  // PAIR: rank in the pair, the pair's index among all pairs, and the number of pairs.
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const int unit = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int units = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) { mbar_init(&full_bar[s], 1); mbar_init(&empty_bar[s], 1); }
    // PAIR: one arrival per epilogue warp of both CTAs, on the even CTA's barrier
    const uint32_t acc_empty_count = PAIR ? 2 * kGemmEpiWarps : 32 * kGemmEpiWarps;
    for (int b = 0; b < 2; ++b) { mbar_init(&acc_full[b], 1); mbar_init(&acc_empty[b], acc_empty_count); }
    mbar_init(&drain_bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) { tma_prefetch_desc(&tma_a); tma_prefetch_desc(&tma_b); }
  if (warp == 1) {
    if constexpr (PAIR) { tmem_alloc_pair(&tmem_base_slot, 2 * BN); tmem_relinquish_pair(); }
    else { tmem_alloc(&tmem_base_slot, 2 * BN); tmem_relinquish(); }
  }
  tc_fence_before();
  if constexpr (PAIR) cluster_sync();
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_slot;
  volatile int* abort = &abort_flag;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = unit; tile < p.num_tiles && ok; tile += units) {
        const int tm = tile / p.tiles_n, tn = tile % p.tiles_n;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort)) { ok = false; break; }
          uint8_t* sa = smem + stage * S::kStage;
          uint8_t* sb = sa + S::kA;
          if constexpr (PAIR) {
            // both CTAs' halves count on the even CTA's barrier, which expects both
            const uint32_t bar = cluster_addr(&full_bar[stage], 0);
            if (rank == 0) mbar_arrive_expect_tx(&full_bar[stage], 2 * S::kStage);
#pragma unroll
            for (int at = 0; at < KATOMS; ++at) {
              const int kx = kb * S::kBK + at * kGemmAtom;
              tma_load_2d_pair(sa + at * S::kAtomA, &tma_a, bar, kx, tm * kTileM + static_cast<int>(rank) * kGemmBM);
              tma_load_2d_pair(sb + at * S::kAtomB, &tma_b, bar, kx, tn * BN + static_cast<int>(rank) * (BN / 2));
            }
          } else {
            mbar_arrive_expect_tx(&full_bar[stage], S::kStage);
#pragma unroll
            for (int at = 0; at < KATOMS; ++at) {
              const int kx = kb * S::kBK + at * kGemmAtom;
              tma_load_2d(sa + at * S::kAtomA, &tma_a, &full_bar[stage], kx, tm * kGemmBM);
              tma_load_2d(sb + at * S::kAtomB, &tma_b, &full_bar[stage], kx, tn * BN);
            }
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      if (!ok) {
        // Aborted: give the loads already issued time to land before the CTA can exit.
        for (int i = 0; i < 1000; ++i) __nanosleep(1000);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (lane 0)
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = idesc_i8(kTileM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int tile = unit; tile < p.num_tiles && ok; tile += units, ++local) {
        const int buf = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        const bool drained = PAIR ? mbar_wait_cluster(&acc_empty[buf], acc_phase ^ 1, abort)
                                  : mbar_wait(&acc_empty[buf], acc_phase ^ 1, abort);
        if (!drained) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * S::kStage);
          const uint32_t sb = sa + S::kA;
#pragma unroll
          for (int k = 0; k < S::kBK / 32; ++k) {
            const int at = k / 4, off = (k % 4) * 32;      // atom, then 32-byte step inside its rows
            const uint64_t ad = smem_desc(sa + at * S::kAtomA + off, 16, 1024);
            const uint64_t bd = smem_desc(sb + at * S::kAtomB + off, 16, 1024);
            if constexpr (PAIR) mma_i8_ss_pair(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
            else mma_i8_ss(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          if constexpr (PAIR) {
            mma_commit_pair_both(&empty_bar[stage]);
            if (kb == p.num_kb - 1) mma_commit_pair_both(&acc_full[buf]);
          } else {
            mma_commit(&empty_bar[stage]);
            if (kb == p.num_kb - 1) mma_commit(&acc_full[buf]);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // Every MMA issued above has completed once this commit lands.
      if constexpr (PAIR) mma_commit_pair(&drain_bar);
      else mma_commit(&drain_bar);
      mbar_wait(&drain_bar, 0, nullptr, 1000000);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ epilogue (8 warps)
    const int ew = warp - 2;
    const int quarter = warp & 3;               // TMEM lane quarter this warp may access
    const int half = ew >> 2;                   // which half of the tile's columns
    const int row_in_tile = quarter * 32 + lane;
    float* my_sw = col_sw[ew];
    float* my_bias = col_bias[ew];
    float* my_gate = col_gate[GATED ? ew : 0];
    int local = 0;
    for (int tile = unit; tile < p.num_tiles; tile += units, ++local) {
      const int tm = tile / p.tiles_n, tn = tile % p.tiles_n;
      const int buf = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      const int ncol0 = tn * BN + half * kHalf;         // first output column of this warp
      if (OUT != kOutI32) {
        // Stage this warp's column scales (and bias) in shared memory: broadcast reads below.
        __syncwarp();
        for (int i = lane; i < kHalf; i += 32) {
          const int n = ncol0 + i;
          my_sw[i] = n < p.N ? p.sw[n] : 0.0f;
          if (HAS_BIAS) my_bias[i] = n < p.N ? bias_at<OUT>(p.bias, n) : 0.0f;
          if (GATED) my_gate[i] = n < p.N ? bias_at<OUT>(p.gate, n) : 0.0f;
        }
        __syncwarp();
      }
      bool ok = mbar_wait(&acc_full[buf], acc_phase, abort);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const int row = tm * kTileM + static_cast<int>(rank) * kGemmBM + row_in_tile;
      const bool row_ok = row < p.M;
      const float sxr = (OUT != kOutI32 && row_ok) ? p.sx[row] : 0.0f;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + buf * BN + half * kHalf;
      // output tile origin: with column blocks the tile lies inside one block (col_block % BN == 0)
      int64_t blk_off = 0;
      int col_base = 0;                                   // first column of the tile's block
      if (p.col_block > 0) {
        const int64_t blk = static_cast<int64_t>(tn * BN) / p.col_block;
        blk_off = blk * p.block_stride;
        col_base = static_cast<int>(blk * p.col_block);
      }
      const int64_t out_off = static_cast<int64_t>(row) * p.ldo + blk_off;
      const int row0w = row - lane;                       // this warp's first row
#pragma unroll 1
      for (int c = 0; c < kHalf; c += 32) {
        uint32_t r[32];
        tmem_ld32(taddr + c, r);
        tmem_wait_ld();
        const int col0 = ncol0 + c;
        if (col0 >= p.N) continue;                        // warp-uniform
        if (OUT != kOutI32 && col0 + 32 <= p.N && p.out_vec && (!GATED || p.res_vec)) {
          // Whole 32-column chunk (warp-uniform): the warp moves its 32 x 32 block through shared
          // memory so that each 16-byte global access instruction covers 8 rows' full 64-byte
          // segments (lane l: row 8 it + l / 4, 16 bytes l % 4) instead of one 16-byte piece of
          // each of 32 rows. Unit (row rr, 16 bytes k) sits at rr * 4 + (k ^ (rr / 2 % 4)): both
          // the row-wise and the column-wise accesses then spread over all banks.
          uint4* tile = epi_tile[ew];
          auto unit = [](int rr, int k) { return rr * 4 + (k ^ ((rr >> 1) & 3)); };
          uint32_t res[16];
          if (GATED) {
#pragma unroll
            for (int it = 0; it < 4; ++it) {
              const int rr = 8 * it + (lane >> 2), k = lane & 3;
              const int grow = row0w + rr;
              uint4 v = make_uint4(0, 0, 0, 0);
              if (grow < p.M)
                v = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(p.residual) +
                                                    static_cast<int64_t>(grow) * p.ldr + col0 + 8 * k);
              tile[unit(rr, k)] = v;
            }
            __syncwarp();
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint4 u = tile[unit(lane, k)];
              res[4 * k] = u.x; res[4 * k + 1] = u.y; res[4 * k + 2] = u.z; res[4 * k + 3] = u.w;
            }
            __syncwarp();
          }
          uint32_t w[16];
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            const float4 s4 = *reinterpret_cast<const float4*>(my_sw + c + j);
            float4 b4 = make_float4(0.f, 0.f, 0.f, 0.f);
            if (HAS_BIAS) b4 = *reinterpret_cast<const float4*>(my_bias + c + j);
            float y0 = epi_value<OUT, HAS_BIAS, GELU>(r[j], sxr, s4.x, b4.x);
            float y1 = epi_value<OUT, HAS_BIAS, GELU>(r[j + 1], sxr, s4.y, b4.y);
            float y2 = epi_value<OUT, HAS_BIAS, GELU>(r[j + 2], sxr, s4.z, b4.z);
            float y3 = epi_value<OUT, HAS_BIAS, GELU>(r[j + 3], sxr, s4.w, b4.w);
            if (GATED) {
              const float4 g4 = *reinterpret_cast<const float4*>(my_gate + c + j);
              y0 = gated_residual<OUT>(res[j / 2] & 0xFFFFu, g4.x, y0);
              y1 = gated_residual<OUT>(res[j / 2] >> 16, g4.y, y1);
              y2 = gated_residual<OUT>(res[j / 2 + 1] & 0xFFFFu, g4.z, y2);
              y3 = gated_residual<OUT>(res[j / 2 + 1] >> 16, g4.w, y3);
            }
            w[j / 2] = OUT == kOutBF16 ? pack_bf16x2(y0, y1) : pack_f16x2(y0, y1);
            w[j / 2 + 1] = OUT == kOutBF16 ? pack_bf16x2(y2, y3) : pack_f16x2(y2, y3);
          }
#pragma unroll
          for (int k = 0; k < 4; ++k) tile[unit(lane, k)] = make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
          __syncwarp();
#pragma unroll
          for (int it = 0; it < 4; ++it) {
            const int rr = 8 * it + (lane >> 2), k = lane & 3;
            const int grow = row0w + rr;
            if (grow < p.M)
              *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.out) + static_cast<int64_t>(grow) * p.ldo +
                                        blk_off + (col0 - col_base) + 8 * k) = tile[unit(rr, k)];
          }
          __syncwarp();
          continue;
        }
        if (!row_ok) continue;
        if (OUT == kOutI32) {
          int32_t* dst = reinterpret_cast<int32_t*>(p.out) + out_off + (col0 - col_base);
          if (col0 + 32 <= p.N && p.out_vec) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
              *reinterpret_cast<uint4*>(dst + j) = make_uint4(r[j], r[j + 1], r[j + 2], r[j + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (col0 + j < p.N) dst[j] = static_cast<int32_t>(r[j]);
          }
        } else {
          uint16_t* dst = reinterpret_cast<uint16_t*>(p.out) + out_off + (col0 - col_base);
          uint32_t w[16];
          uint32_t res[16];
          if (GATED) {
            const uint16_t* rp = reinterpret_cast<const uint16_t*>(p.residual) + static_cast<int64_t>(row) * p.ldr + col0;
            if (col0 + 32 <= p.N && p.res_vec) {
#pragma unroll
              for (int j = 0; j < 16; j += 4) {
                const uint4 u = *reinterpret_cast<const uint4*>(rp + 2 * j);
                res[j] = u.x; res[j + 1] = u.y; res[j + 2] = u.z; res[j + 3] = u.w;
              }
            } else {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const uint32_t lo = col0 + 2 * j < p.N ? rp[2 * j] : 0u;
                const uint32_t hi = col0 + 2 * j + 1 < p.N ? rp[2 * j + 1] : 0u;
                res[j] = lo | (hi << 16);
              }
            }
          }
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            const float4 s4 = *reinterpret_cast<const float4*>(my_sw + c + j);
            float4 b4 = make_float4(0.f, 0.f, 0.f, 0.f);
            if (HAS_BIAS) b4 = *reinterpret_cast<const float4*>(my_bias + c + j);
            float y0 = epi_value<OUT, HAS_BIAS, GELU>(r[j], sxr, s4.x, b4.x);
            float y1 = epi_value<OUT, HAS_BIAS, GELU>(r[j + 1], sxr, s4.y, b4.y);
            float y2 = epi_value<OUT, HAS_BIAS, GELU>(r[j + 2], sxr, s4.z, b4.z);
            float y3 = epi_value<OUT, HAS_BIAS, GELU>(r[j + 3], sxr, s4.w, b4.w);
            if (GATED) {
              const float4 g4 = *reinterpret_cast<const float4*>(my_gate + c + j);
              y0 = gated_residual<OUT>(res[j / 2] & 0xFFFFu, g4.x, y0);
              y1 = gated_residual<OUT>(res[j / 2] >> 16, g4.y, y1);
              y2 = gated_residual<OUT>(res[j / 2 + 1] & 0xFFFFu, g4.z, y2);
              y3 = gated_residual<OUT>(res[j / 2 + 1] >> 16, g4.w, y3);
            }
            w[j / 2] = OUT == kOutBF16 ? pack_bf16x2(y0, y1) : pack_f16x2(y0, y1);
            w[j / 2 + 1] = OUT == kOutBF16 ? pack_bf16x2(y2, y3) : pack_f16x2(y2, y3);
          }
          if (col0 + 32 <= p.N && p.out_vec) {
#pragma unroll
            for (int j = 0; j < 16; j += 4)
              *reinterpret_cast<uint4*>(dst + 2 * j) = make_uint4(w[j], w[j + 1], w[j + 2], w[j + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (col0 + j < p.N) dst[j] = static_cast<uint16_t>(w[j / 2] >> (16 * (j & 1)));
          }
        }
      }
      tc_fence_before();
      if constexpr (PAIR) {
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(cluster_addr(&acc_empty[buf], 0));
      } else {
        mbar_arrive(&acc_empty[buf]);
      }
    }
  }

  tc_fence_before();
  if constexpr (PAIR) cluster_sync();
  else __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem_base, 2 * BN);
    else tmem_dealloc(tmem_base, 2 * BN);
  }
}

// Standalone rescale of an int32 accumulator (the reference's `rescale`,
// src/diffucore/models/_int8.py:313-323) for callers that hold an int_mm result; the GEMM
// applies the same epilogue in place. Grid-stride over rows, 8 columns per thread step.
template <int OUT>
__global__ void __launch_bounds__(256)
rescale_kernel(const int32_t* __restrict__ acc, int64_t lda, const float* __restrict__ sx,
               const float* __restrict__ sw, const void* bias, void* out, int64_t ldo, int M, int N) {
  const bool has_bias = bias != nullptr;
  for (int64_t row = blockIdx.x; row < M; row += gridDim.x) {
    const float sxr = sx[row];
    const int32_t* a = acc + row * lda;
    uint16_t* dst = reinterpret_cast<uint16_t*>(out) + row * ldo;
    for (int n = threadIdx.x; n < N; n += blockDim.x) {
      const float bn = has_bias ? bias_at<OUT>(bias, n) : 0.0f;
      const float y = has_bias ? epi_value<OUT, true, 0>(static_cast<uint32_t>(a[n]), sxr, sw[n], bn)
                               : epi_value<OUT, false, 0>(static_cast<uint32_t>(a[n]), sxr, sw[n], bn);
      if (OUT == kOutBF16) {
        __nv_bfloat16 h = __float2bfloat16_rn(y);
        dst[n] = *reinterpret_cast<uint16_t*>(&h);
      } else {
        __half h = __float2half_rn(y);
        dst[n] = *reinterpret_cast<uint16_t*>(&h);
      }
    }
  }
}

}  // namespace dc
