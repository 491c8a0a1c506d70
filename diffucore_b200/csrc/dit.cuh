// Producer-side glue of a FLUX-architecture DiT block, fused around the W8A8 linears and the
// INT8 attention (HBM-bound, one read and one write of each row):
//
//  * ln_mod_quant_kernel: LayerNorm (no affine, eps 1e-6) -> AdaLN modulation -> optional
//    256-wide rotation -> per-row int8 codes. It replaces the torch sequence
//        x_mod = (1 + mod.scale) * norm(x) + mod.shift        (src/diffucore/models/flux_dit.py:282,
//                                                              :287, :328)
//    followed by `Int8Linear.forward`'s `quantize_activation` (src/diffucore/models/_int8.py:299-310),
//    so the modulated activation never exists in HBM. Each torch op of that sequence rounds to the
//    model dtype; the kernel rounds at the same points: n = dtype(LN(x)), a = dtype(1 + scale),
//    t = dtype(a * n), y = dtype(t + shift).
//  * qk_norm_rope_kernel: per-head RMSNorm of q and k with their learned scales, then the axial
//    RoPE rotation, in place on the packed qkv rows (flux_dit.py:129-151 `RMSNorm`/`QKNorm`,
//    :179-184 `apply_rope`). Rounding points as in torch: dtype(x * rrms), dtype(that * scale),
//    RoPE in fp32 as two products and a sum, then dtype.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>
#include <type_traits>
#include "sm100.cuh"
#include "quant.cuh"
#include "gemm.cuh"

namespace dc {

template <typename T>
__device__ __forceinline__ float rnd(float x) { return Vec8<T>::round_trip(x); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Warp per row, K <= 32 * 8 * VPT, K % 8 == 0 (K % 256 == 0 with GROUP). Rows of batch element b
// (b = row / rows_per_mod) use shift/scale + b * mod_ld.
template <typename T, int VPT, bool GROUP>
__global__ void __launch_bounds__(128)
ln_mod_quant_kernel(const T* __restrict__ x, int64_t M, int K, int64_t ldx, const T* __restrict__ shift,
                    const T* __restrict__ scale, int64_t rows_per_mod, int64_t mod_ld, int8_t* __restrict__ q,
                    float* __restrict__ s, int full_div) {
  const int lane = threadIdx.x & 31;
  const int nvec = K >> 3;
  const float inv_k = 1.0f / static_cast<float>(K);
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); row < M;
       row += warps) {
    const T* xr = x + row * ldx;
    float v[VPT][8];
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = lane + 32 * i;
      if (vi < nvec) {
        Vec8<T>::load(xr + vi * 8, v[i]);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = 0.0f;
      }
    }
    // mean and biased variance in fp32 (two passes over registers, four independent sum chains)
    float a4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int i = 0; i < VPT; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) a4[j & 3] = __fadd_rn(a4[j & 3], v[i][j]);
    const float mean = __fmul_rn(warp_sum(__fadd_rn(__fadd_rn(a4[0], a4[1]), __fadd_rn(a4[2], a4[3]))), inv_k);
#pragma unroll
    for (int c = 0; c < 4; ++c) a4[c] = 0.0f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = lane + 32 * i;
      if (vi < nvec) {
#pragma unroll
        for (int j = 0; j < 8; ++j) { const float d = __fsub_rn(v[i][j], mean); a4[j & 3] = __fmaf_rn(d, d, a4[j & 3]); }
      }
    }
    const float var = __fmul_rn(warp_sum(__fadd_rn(__fadd_rn(a4[0], a4[1]), __fadd_rn(a4[2], a4[3]))), inv_k);
    const float rstd = rsqrtf(__fadd_rn(var, 1e-6f));
    const int64_t b = row / rows_per_mod;
    const T* shr = shift + b * mod_ld;
    const T* scr = scale + b * mod_ld;
    float am4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = lane + 32 * i;
      if (vi < nvec) {
        float sh[8], sc[8];
        Vec8<T>::load(shr + vi * 8, sh);
        Vec8<T>::load(scr + vi * 8, sc);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float n = rnd<T>(__fmul_rn(__fsub_rn(v[i][j], mean), rstd));
          const float a = rnd<T>(__fadd_rn(1.0f, sc[j]));
          v[i][j] = rnd<T>(__fadd_rn(rnd<T>(__fmul_rn(a, n)), sh[j]));
        }
      }
      // the 32 lanes at one i hold one 256-wide group; lanes past the row end hold zeros
      if (GROUP) hadamard256_warp(v[i], rot_order_for_width(K));
#pragma unroll
      for (int j = 0; j < 8; ++j) am4[j & 3] = fmaxf(am4[j & 3], fabsf(v[i][j]));
    }
    float am = fmaxf(fmaxf(am4[0], am4[1]), fmaxf(am4[2], am4[3]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    const float sc = row_scale(am, full_div);
    const float inv = __fdiv_rn(1.0f, sc);
    int8_t* qr = q + row * static_cast<int64_t>(K);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = lane + 32 * i;
      if (vi < nvec) *reinterpret_cast<uint2*>(qr + vi * 8) = quant8(v[i], sc, inv, full_div);
    }
    if (lane == 0) s[row] = sc;
  }
}

struct QkNormRopeParams {
  void* qkv;                 // row r, head h: q at qkv + r*ld_row + q_off + h*128, k at + k_off
  int64_t L, H, ld_row, q_off, k_off;
  const void* q_scale[2];    // per-dim RMSNorm scales: [0] for rows < split_row, [1] for the rest
  const void* k_scale[2];
  int64_t split_row;
  const float* pe;           // [L, 64, 2, 2] fp32: rows {cos, -sin}, {sin, cos} per rotary pair
  int64_t pe_row0;           // row r of qkv uses pe row pe_row0 + r
  // Optional Q codes for the INT8 attention in the reference quant mode (one sequence): head h of
  // row r gets codes q_codes[(h * q_lpad + r) * 128 ..] and scale q_rscale[h * q_lpad + r], with
  // q_token_quant_kernel's arithmetic; rows [L, q_lpad) get zero codes and scales. write_q = 0
  // leaves the normed, rotated q out of qkv (only the codes are needed then).
  int8_t* q_codes = nullptr;
  float* q_rscale = nullptr;
  int64_t q_lpad = 0;
  int write_q = 1;
};

// One warp per (row, head, q|k) vector (lane holds elements 4 lane .. 4 lane + 3 = rotary pairs
// 2 lane, 2 lane + 1); a warp loads its kRopeBatch vectors before computing any.
template <typename T>
__device__ __forceinline__ void rms_rope4(uint2& raw, const T* scl, float4 f0, float4 f1) {
  const uint2 sraw = *reinterpret_cast<const uint2*>(scl);
  float x[4], g[4];
  {
    float tmp[8], stmp[8];
    Vec8<T>::from_raw(make_uint4(raw.x, raw.y, 0u, 0u), tmp);
    Vec8<T>::from_raw(make_uint4(sraw.x, sraw.y, 0u, 0u), stmp);
#pragma unroll
    for (int j = 0; j < 4; ++j) { x[j] = tmp[j]; g[j] = stmp[j]; }
  }
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < 4; ++j) ss = __fadd_rn(ss, __fmul_rn(x[j], x[j]));
  const float rrms = rsqrtf(__fadd_rn(__fmul_rn(warp_sum(ss), 1.0f / 128.0f), 1e-6f));
  float y[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) y[j] = rnd<T>(__fmul_rn(rnd<T>(__fmul_rn(x[j], rrms)), g[j]));
  // pair 0: (y0, y1) with f0 = {f00, f01, f10, f11}; pair 1: (y2, y3) with f1
  const float o0 = rnd<T>(__fadd_rn(__fmul_rn(f0.x, y[0]), __fmul_rn(f0.y, y[1])));
  const float o1 = rnd<T>(__fadd_rn(__fmul_rn(f0.z, y[0]), __fmul_rn(f0.w, y[1])));
  const float o2 = rnd<T>(__fadd_rn(__fmul_rn(f1.x, y[2]), __fmul_rn(f1.y, y[3])));
  const float o3 = rnd<T>(__fadd_rn(__fmul_rn(f1.z, y[2]), __fmul_rn(f1.w, y[3])));
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    raw.x = pack_bf16x2(o0, o1);
    raw.y = pack_bf16x2(o2, o3);
  } else {
    raw.x = pack_f16x2(o0, o1);
    raw.y = pack_f16x2(o2, o3);
  }
}

constexpr int kRopeWarps = 8;
constexpr int kRopeBatch = 6;     // vectors per warp loaded together

template <typename T>
__global__ void __launch_bounds__(32 * kRopeWarps)
qk_norm_rope_kernel(const QkNormRopeParams p) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nvec = static_cast<int>(2 * p.H);
  if (p.q_codes != nullptr) {
    // padding rows of the Q codes: zero, as the per-token quantizer leaves them
    for (int64_t row = p.L + blockIdx.x; row < p.q_lpad; row += gridDim.x)
      for (int h = warp; h < p.H; h += kRopeWarps) {
        *reinterpret_cast<uint32_t*>(p.q_codes + (h * p.q_lpad + row) * 128 + lane * 4) = 0u;
        if (lane == 0) p.q_rscale[h * p.q_lpad + row] = 0.0f;
      }
  }
  // (row, vector) items, item = row * nvec + v, dealt to the warps of the grid in turn: few heads
  // per row (a sequence-parallel split leaves 3 of 24) fill the warps as well as many do.
  const uint32_t n_items = static_cast<uint32_t>(p.L) * static_cast<uint32_t>(nvec);   // < 2^31 (host)
  const uint32_t nw = gridDim.x * kRopeWarps;
  for (uint32_t i0 = blockIdx.x * kRopeWarps + warp; i0 < n_items; i0 += nw * kRopeBatch) {
    uint2 raw[kRopeBatch];
    uint32_t rows[kRopeBatch];
    int vs[kRopeBatch];
#pragma unroll
    for (int b = 0; b < kRopeBatch; ++b) {
      const uint32_t item = i0 + b * nw;
      rows[b] = item / static_cast<uint32_t>(nvec);
      vs[b] = static_cast<int>(item - rows[b] * static_cast<uint32_t>(nvec));
      if (item < n_items)
        raw[b] = *reinterpret_cast<const uint2*>(static_cast<const T*>(p.qkv) + rows[b] * p.ld_row + lane * 4 +
                                                 ((vs[b] & 1) ? p.k_off : p.q_off) + (vs[b] >> 1) * 128);
    }
#pragma unroll
    for (int b = 0; b < kRopeBatch; ++b) {
      if (i0 + b * nw >= n_items) break;             // warp-uniform; later items are further out
      const int64_t row = rows[b];
      const int v = vs[b];
      const float4* pe4 = reinterpret_cast<const float4*>(p.pe + (p.pe_row0 + row) * 256 + lane * 8);
      const bool first = row < p.split_row;
      const bool is_q = (v & 1) == 0;
      const T* scl = static_cast<const T*>(is_q ? (first ? p.q_scale[0] : p.q_scale[1])
                                                : (first ? p.k_scale[0] : p.k_scale[1])) + lane * 4;
      rms_rope4<T>(raw[b], scl, pe4[0], pe4[1]);
      T* dst = static_cast<T*>(p.qkv) + row * p.ld_row + lane * 4 + (is_q ? p.q_off : p.k_off) + (v >> 1) * 128;
      if (!is_q || p.write_q) *reinterpret_cast<uint2*>(dst) = raw[b];
      if (is_q && p.q_codes != nullptr) {
        // the per-token Q codes of this head (q_token_quant_kernel's arithmetic on the rounded
        // values just stored): amax over the 128 channels, codes rn(x * 127 / amax)
        float f[8];
        Vec8<T>::from_raw(make_uint4(raw[b].x, raw[b].y, 0u, 0u), f);
        float amax = fmaxf(fmaxf(fabsf(f[0]), fabsf(f[1])), fmaxf(fabsf(f[2]), fabsf(f[3])));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float inv = amax > 0.f ? __fdiv_rn(127.f, amax) : 0.f;
        uint32_t w = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) w |= code_byte(__fmul_rn(f[i], inv)) << (8 * i);
        const int64_t qrow = static_cast<int64_t>(v >> 1) * p.q_lpad + row;
        *reinterpret_cast<uint32_t*>(p.q_codes + qrow * 128 + lane * 4) = w;
        if (lane == 0) p.q_rscale[qrow] = __fdiv_rn(amax, 127.f);
      }
    }
  }
}

}  // namespace dc
