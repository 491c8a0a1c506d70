// Per-row symmetric int8 quantizer with optional 256-wide ConvRot (Hadamard) rotation and
// optional GELU applied first. HBM-bound: one read of the row, one int8 write, one scale.
//
// Arithmetic follows the reference's torch-op path bit for bit
// (src/diffucore/models/_int8.py:87-97 `_quantize_rows`, :393-397 `_store_quantized`):
//   scale = max(amax / 127, 1e-30)     (IEEE fp32 division)
//   q     = clamp(rint(x / scale), -128, 127)   (IEEE division, round half to even)
// The rotation is the radix-4 butterfly of `_hadamard_rows` (_int8.py:364-372): for each base-4
// digit of the in-group index, most significant first, y = S - 2 * x[digit -> 3 - digit] with
// S = (x[d=0] + x[d=1]) + (x[d=2] + x[d=3]); then y * 0.0625. That summation order is this
// library's definition; the CPU oracle restates it.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>
#include "sm100.cuh"

namespace dc {

enum GeluMode : int { kGeluNone = 0, kGeluErf = 1, kGeluTanh = 2 };

template <typename T> struct Vec8;
template <> struct Vec8<__nv_bfloat16> {
  __device__ static void load(const __nv_bfloat16* p, float (&f)[8]) {
    uint4 u = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) { float2 t = __bfloat1622float2(h[i]); f[2 * i] = t.x; f[2 * i + 1] = t.y; }
  }
  __device__ static float one(const __nv_bfloat16* p) { return __bfloat162float(*p); }
  __device__ static float round_trip(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
};
template <> struct Vec8<__half> {
  __device__ static void load(const __half* p, float (&f)[8]) {
    uint4 u = *reinterpret_cast<const uint4*>(p);
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) { float2 t = __half22float2(h[i]); f[2 * i] = t.x; f[2 * i + 1] = t.y; }
  }
  __device__ static float one(const __half* p) { return __half2float(*p); }
  __device__ static float round_trip(float x) { return __half2float(__float2half_rn(x)); }
};
template <> struct Vec8<float> {
  __device__ static void load(const float* p, float (&f)[8]) {
    float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  }
  __device__ static float one(const float* p) { return *p; }
  __device__ static float round_trip(float x) { return x; }
};

// GELU of a value already in the model dtype, rounded back to that dtype (the reference's
// `_gelu`, _int8.py:432-434, and FLUX's tanh form, nn.GELU(approximate="tanh")).
template <typename T>
__device__ __forceinline__ float gelu_dtype(float h, int mode) {
  if (mode == kGeluErf) {
    const float t = __fmul_rn(h, 0.7071067811865476f);
    const float e = __fadd_rn(1.0f, erff(t));
    return Vec8<T>::round_trip(__fmul_rn(__fmul_rn(0.5f, h), e));
  }
  if (mode == kGeluTanh) {
    // 0.5 * h * (1 + tanh(sqrt(2/pi) * (h + 0.044715 * h^3)))
    const float h3 = __fmul_rn(__fmul_rn(h, h), h);
    const float inner = __fmul_rn(0.7978845608028654f, __fadd_rn(h, __fmul_rn(0.044715f, h3)));
    const float e = __fadd_rn(1.0f, tanhf(inner));
    return Vec8<T>::round_trip(__fmul_rn(__fmul_rn(0.5f, h), e));
  }
  return h;
}

__device__ __forceinline__ float quad_sum(float a0, float a1, float a2, float a3) {
  return __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3));
}

// One radix-4 stage across lanes: the digit lives in lane bits (xor masks m_lo, m_hi);
// `flip_mask` = m_lo | m_hi selects the lane holding digit 3 - d.
__device__ __forceinline__ float hstage_lanes(float x, int m_lo, int m_hi) {
  const float a = __fadd_rn(x, __shfl_xor_sync(0xffffffffu, x, m_lo));   // x[d] + x[d^1]
  const float s = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, m_hi));   // (x0+x1)+(x2+x3) in every lane
  const float f = __shfl_xor_sync(0xffffffffu, x, m_lo | m_hi);          // x[3 - d]
  return __fsub_rn(s, __fmul_rn(2.0f, f));
}

// Rotate the 8 values a lane holds; 32 lanes of a warp hold one 256-wide group, element
// e = lane * 8 + j. Digits: d0 = j & 3, d1 = ((lane & 1) << 1) | (j >> 2), d2 = (lane >> 1) & 3,
// d3 = lane >> 3. Stage order d3, d2, d1, d0 (most significant first).
__device__ __forceinline__ void hadamard256_warp(float (&x)[8]) {
  // d3: lane bits 3 and 4.
#pragma unroll
  for (int j = 0; j < 8; ++j) x[j] = hstage_lanes(x[j], 8, 16);
  // d2: lane bits 1 and 2.
#pragma unroll
  for (int j = 0; j < 8; ++j) x[j] = hstage_lanes(x[j], 2, 4);
  // d1: low bit is j bit 2 (in-thread), high bit is lane bit 0.
  {
    float y[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float lo = (j < 4) ? __fadd_rn(x[j], x[j + 4]) : __fadd_rn(x[j - 4], x[j]);   // x[d1=2h] + x[d1=2h+1]
      const float lo_other = __shfl_xor_sync(0xffffffffu, lo, 1);
      const bool low_half = (threadIdx.x & 1) == 0;   // this lane holds d1 in {0, 1}
      const float s = low_half ? __fadd_rn(lo, lo_other) : __fadd_rn(lo_other, lo);
      const float f = __shfl_xor_sync(0xffffffffu, x[j ^ 4], 1);                      // x[3 - d1]
      y[j] = __fsub_rn(s, __fmul_rn(2.0f, f));
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) x[j] = y[j];
  }
  // d0: j bits 0 and 1, all in-thread.
  {
    float y[8];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float s = quad_sum(x[4 * h], x[4 * h + 1], x[4 * h + 2], x[4 * h + 3]);
#pragma unroll
      for (int d = 0; d < 4; ++d) y[4 * h + d] = __fsub_rn(s, __fmul_rn(2.0f, x[4 * h + (3 - d)]));
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) x[j] = __fmul_rn(y[j], 0.0625f);
  }
}

__device__ __forceinline__ int8_t quant_code(float x, float scale) {
  float t = rintf(__fdiv_rn(x, scale));
  t = fminf(fmaxf(t, -128.0f), 127.0f);
  return static_cast<int8_t>(static_cast<int>(t));
}

constexpr int kQuantThreads = 128;

// Vector path: K % 8 == 0, ldx % 8 == 0 (elements), x 16-byte aligned. One CTA per row
// (grid-stride). Each thread holds up to VPT vectors of 8 elements. `group` is 0 or 256.
template <typename T, int VPT>
__global__ void __launch_bounds__(kQuantThreads)
quant_rows_kernel(const T* __restrict__ x, int64_t M, int K, int64_t ldx, int group, int gelu,
                  int8_t* __restrict__ q, float* __restrict__ s) {
  __shared__ float red[kQuantThreads / 32];
  const int tid = threadIdx.x;
  const int nvec = K >> 3;
  for (int64_t row = blockIdx.x; row < M; row += gridDim.x) {
    const T* xr = x + row * ldx;
    float v[VPT][8];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = tid + i * kQuantThreads;
      if (vi < nvec) {
        Vec8<T>::load(xr + vi * 8, v[i]);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = 0.0f;
      }
      if (gelu != kGeluNone) {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = gelu_dtype<T>(v[i][j], gelu);
      }
      // A 256-group is 32 consecutive vectors = the 32 lanes of one warp at one i. Groups
      // past the row end hold zeros and are discarded; every lane joins the shuffles.
      if (group) hadamard256_warp(v[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[i][j]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((tid & 31) == 0) red[tid >> 5] = amax;
    __syncthreads();
    amax = red[0];
#pragma unroll
    for (int w = 1; w < kQuantThreads / 32; ++w) amax = fmaxf(amax, red[w]);
    __syncthreads();
    const float scale = fmaxf(__fdiv_rn(amax, 127.0f), 1e-30f);
    int8_t* qr = q + row * static_cast<int64_t>(K);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = tid + i * kQuantThreads;
      if (vi < nvec) {
        uint32_t w0 = 0, w1 = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          w0 |= static_cast<uint32_t>(static_cast<uint8_t>(quant_code(v[i][j], scale))) << (8 * j);
          w1 |= static_cast<uint32_t>(static_cast<uint8_t>(quant_code(v[i][j + 4], scale))) << (8 * j);
        }
        *reinterpret_cast<uint2*>(qr + vi * 8) = make_uint2(w0, w1);
      }
    }
    if (tid == 0) s[row] = scale;
  }
}

// Generic path for any K and stride (no rotation): two passes over the row.
template <typename T>
__global__ void __launch_bounds__(kQuantThreads)
quant_rows_scalar_kernel(const T* __restrict__ x, int64_t M, int K, int64_t ldx, int gelu,
                         int8_t* __restrict__ q, float* __restrict__ s) {
  __shared__ float red[kQuantThreads / 32];
  const int tid = threadIdx.x;
  for (int64_t row = blockIdx.x; row < M; row += gridDim.x) {
    const T* xr = x + row * ldx;
    float amax = 0.0f;
    for (int c = tid; c < K; c += kQuantThreads) {
      float t = Vec8<T>::one(xr + c);
      if (gelu != kGeluNone) t = gelu_dtype<T>(t, gelu);
      amax = fmaxf(amax, fabsf(t));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((tid & 31) == 0) red[tid >> 5] = amax;
    __syncthreads();
    amax = red[0];
#pragma unroll
    for (int w = 1; w < kQuantThreads / 32; ++w) amax = fmaxf(amax, red[w]);
    __syncthreads();
    const float scale = fmaxf(__fdiv_rn(amax, 127.0f), 1e-30f);
    int8_t* qr = q + row * static_cast<int64_t>(K);
    for (int c = tid; c < K; c += kQuantThreads) {
      float t = Vec8<T>::one(xr + c);
      if (gelu != kGeluNone) t = gelu_dtype<T>(t, gelu);
      qr[c] = quant_code(t, scale);
    }
    if (tid == 0) s[row] = scale;
  }
}

}  // namespace dc
