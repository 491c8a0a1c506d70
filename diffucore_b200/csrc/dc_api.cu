// C-ABI of the B200 hot path. Plain pointers and sizes in, an int status out (0 = ok);
// dc_last_error() returns the reason of the last non-zero status on the calling thread.
// The library never allocates or frees device memory: callers pass outputs and workspaces.
// Every launch goes on the stream the caller passes; nothing here synchronizes.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <atomic>
#include <mutex>
#include <type_traits>

#include "../../include/diffucore_b200.h"

// Size of the fixed scratch behind dc_attn_int8_fwd_noalloc (32 MiB per GPU).
constexpr size_t kNoAllocScratch = static_cast<size_t>(DC_NOALLOC_SCRATCH_BYTES);
#include "sm100.cuh"
#include "quant.cuh"
#include "rowquant.cuh"
#include "gemm.cuh"
#include "attn.cuh"
#include "dit.cuh"

namespace {

thread_local char g_err[512] = "";

// Division arithmetic of every per-row quantizer launch (DC_QDIV_IEEE / DC_QDIV_FULL), set by
// dc_set_quant_division; read when a launch is enqueued.
std::atomic<int> g_quant_div{DC_QDIV_IEEE};

int quant_full_div() { return g_quant_div.load(std::memory_order_relaxed) == DC_QDIV_FULL ? 1 : 0; }

int fail(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return DC_ERR_INVALID;
}

int cuda_fail(cudaError_t e, const char* what) {
  snprintf(g_err, sizeof(g_err), "%s: %s", what, cudaGetErrorString(e));
  return DC_ERR_CUDA;
}

#define DC_CHECK_LAUNCH(what)                          \
  do {                                                 \
    cudaError_t e_ = cudaGetLastError();               \
    if (e_ != cudaSuccess) return cuda_fail(e_, what); \
  } while (0)

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// rank-N tiled map; dims/strides innermost first, strides in bytes for dims 1..N-1.
int make_map(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base, const uint64_t* dims,
             const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swz) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail("cuTensorMapEncodeTiled is not available from the CUDA driver");
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) return fail("TMA base address is not 16-byte aligned");
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) { d[i] = dims[i]; b[i] = box[i]; e[i] = 1; }
  for (int i = 0; i + 1 < rank; ++i) {
    if (strides_bytes[i] % 16 != 0) return fail("TMA stride %llu bytes is not a multiple of 16",
                                                (unsigned long long)strides_bytes[i]);
    s[i] = strides_bytes[i];
  }
  CUresult r = fn(map, dt, rank, const_cast<void*>(base), d, s, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail("cuTensorMapEncodeTiled failed (CUresult %d)", static_cast<int>(r));
  return DC_OK;
}

int sm_count() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

int check_sm100() {
  int dev = 0, major = 0, minor = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail("no CUDA device");
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (major != 10 || minor != 0) return fail("device is sm_%d%d; this library is built for sm_100a only", major, minor);
  return DC_OK;
}

template <typename K>
int set_smem(K kernel, int bytes) {
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
  return DC_OK;
}

inline int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

// ------------------------------------------------------------------------------ quantizer

// Shared-memory streaming quantizers (rowquant.cuh): K % 256 == 0, 16-bit rows, no GELU.
constexpr int kRowqWarps = 8;

// Rotated rows (group 256) go to the quantizers computing two groups per half-warp with packed
// fp32 operations (rowq_pair_kernel, rowq_cta_pair_kernel): the same codes and scales as the
// one-group kernels, 17-19 % less time at FLUX's 3072- and 15360-wide rows on a B200.
// DC_ROWQ_PAIR=0 selects the one-group kernels (rowq_warp_kernel, rowq_cta_kernel) instead.
bool use_rowq_pair() {
  const char* env = getenv("DC_ROWQ_PAIR");
  return env == nullptr || strcmp(env, "0") != 0;
}

template <typename T, bool LNMOD, bool SEG>
int launch_rowq_pair(const dc::RowSrc& src, int64_t M, int64_t K, const void* shift, const void* scale, int8_t* q,
                     float* s, cudaStream_t st) {
  const int nit2 = static_cast<int>((K / 256 + 3) / 4);
  const size_t smem = (LNMOD ? 2 * K * sizeof(float) : 0) + static_cast<size_t>(kRowqWarps) * 2 * K * sizeof(T) +
                      static_cast<size_t>(kRowqWarps) * 2 * dc::kRotScratch2 * sizeof(float2);
  const int64_t ctas64 = (M + kRowqWarps - 1) / kRowqWarps;
  const int ctas = static_cast<int>(ctas64 < sm_count() ? ctas64 : sm_count());
  const T* sh = static_cast<const T*>(shift);
  const T* sc = static_cast<const T*>(scale);
  const int Ki = static_cast<int>(K);
  int r = DC_OK;
  auto go = [&](auto kernel) {
    r = set_smem(kernel, static_cast<int>(smem));
    if (r == DC_OK) kernel<<<ctas, 32 * kRowqWarps, smem, st>>>(src, M, Ki, sh, sc, q, s);
  };
  if (nit2 <= 1) go(dc::rowq_pair_kernel<T, LNMOD, SEG, 1>);
  else if (nit2 <= 2) go(dc::rowq_pair_kernel<T, LNMOD, SEG, 2>);
  else if (nit2 <= 3) go(dc::rowq_pair_kernel<T, LNMOD, SEG, 3>);
  else go(dc::rowq_pair_kernel<T, LNMOD, SEG, 4>);
  if (r) return r;
  DC_CHECK_LAUNCH("quant_rows launch");
  return DC_OK;
}

// Rows held in registers, one CTA per row (rowq_reg_kernel): the default for rotated 16-bit rows
// and LayerNorm + modulation rows, K % 256 == 0 up to 16384 wide (segmented rows: segments of 256
// columns or more). DC_ROWQ_REG=0 selects the shared-memory streaming kernels below; =2 also
// sends plain (unrotated) rows to it.
int rowq_reg_mode() {
  const char* env = getenv("DC_ROWQ_REG");
  if (env == nullptr) return 1;
  return atoi(env);
}

template <typename T, bool LNMOD, bool ROT, bool SEG, int ORD>
int launch_rowq_reg_ord(const dc::RowSrc& src, int64_t M, int64_t K, const void* shift, const void* scale, int8_t* q,
                        float* s, cudaStream_t st) {
  const int nw = static_cast<int>((K / 256 + 3) / 4);
  const int threads = 32 * nw;
  const size_t smem = static_cast<size_t>(nw) * 4 * dc::kRegBlk * sizeof(float) +
                      (LNMOD ? static_cast<size_t>(2) * 16 * threads * sizeof(float2) : 0);
  auto kernel = dc::rowq_reg_kernel<T, LNMOD, ROT, SEG, ORD>;
  if (int r = set_smem(kernel, static_cast<int>(smem))) return r;
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem);
  if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
  const int64_t cap = static_cast<int64_t>(sm_count()) * (per_sm > 0 ? per_sm : 1);
  const int ctas = static_cast<int>(M < cap ? M : cap);
  kernel<<<ctas, threads, smem, st>>>(src, M, static_cast<int>(K), static_cast<const T*>(shift),
                                      static_cast<const T*>(scale), q, s);
  DC_CHECK_LAUNCH("quant_rows launch");
  return DC_OK;
}

// One kernel per summation order class of the rotation (compile-time stage orders).
template <typename T, bool LNMOD, bool ROT, bool SEG>
int launch_rowq_reg(const dc::RowSrc& src, int64_t M, int64_t K, const void* shift, const void* scale, int8_t* q,
                    float* s, cudaStream_t st) {
  if constexpr (!ROT) return launch_rowq_reg_ord<T, LNMOD, false, SEG, 0>(src, M, K, shift, scale, q, s, st);
  switch (src.rot_order) {
    case dc::kRotOrder256: return launch_rowq_reg_ord<T, LNMOD, ROT, SEG, dc::kRotOrder256>(src, M, K, shift, scale, q, s, st);
    case dc::kRotOrder512: return launch_rowq_reg_ord<T, LNMOD, ROT, SEG, dc::kRotOrder512>(src, M, K, shift, scale, q, s, st);
    case dc::kRotOrder1024: return launch_rowq_reg_ord<T, LNMOD, ROT, SEG, dc::kRotOrder1024>(src, M, K, shift, scale, q, s, st);
    case dc::kRotOrderWide: return launch_rowq_reg_ord<T, LNMOD, ROT, SEG, dc::kRotOrderWide>(src, M, K, shift, scale, q, s, st);
    default: return fail("quant_rows: unknown rotation order %d", src.rot_order);
  }
}

template <typename T, bool GROUP, bool LNMOD, bool SEG>
int launch_rowq_warp(const dc::RowSrc& src, int64_t M, int64_t K, const void* shift, const void* scale, int8_t* q,
                     float* s, cudaStream_t st) {
  if constexpr (LNMOD && !SEG) {
    if (rowq_reg_mode() != 0) return launch_rowq_reg<T, true, GROUP, false>(src, M, K, shift, scale, q, s, st);
  }
  if constexpr (GROUP && !(LNMOD && SEG)) {
    if (use_rowq_pair()) return launch_rowq_pair<T, LNMOD, SEG>(src, M, K, shift, scale, q, s, st);
  }
  const int nit = static_cast<int>((K / 256 + 1) / 2);
  const size_t smem = (LNMOD ? 2 * K * sizeof(T) : 0) + static_cast<size_t>(kRowqWarps) * 2 * K * sizeof(T) +
                      static_cast<size_t>(kRowqWarps) * 2 * dc::kRotScratch * sizeof(float);
  const int64_t ctas64 = (M + kRowqWarps - 1) / kRowqWarps;
  const int ctas = static_cast<int>(ctas64 < sm_count() ? ctas64 : sm_count());
  const T* sh = static_cast<const T*>(shift);
  const T* sc = static_cast<const T*>(scale);
  const int Ki = static_cast<int>(K);
  int r = DC_OK;
  auto go = [&](auto kernel) {
    r = set_smem(kernel, static_cast<int>(smem));
    if (r == DC_OK) kernel<<<ctas, 32 * kRowqWarps, smem, st>>>(src, M, Ki, sh, sc, q, s);
  };
  if (nit <= 2) go(dc::rowq_warp_kernel<T, GROUP, LNMOD, SEG, 2>);
  else if (nit <= 4) go(dc::rowq_warp_kernel<T, GROUP, LNMOD, SEG, 4>);
  else if (nit <= 6) go(dc::rowq_warp_kernel<T, GROUP, LNMOD, SEG, 6>);
  else go(dc::rowq_warp_kernel<T, GROUP, LNMOD, SEG, 8>);
  if (r) return r;
  DC_CHECK_LAUNCH("quant_rows launch");
  return DC_OK;
}

template <typename T, bool SEG>
int launch_rowq_cta_pair(const dc::RowSrc& src, int64_t M, int64_t K, int8_t* q, float* s, cudaStream_t st) {
  const int nit2 = static_cast<int>((K / 256 + 31) / 32);
  const size_t smem = 2 * K * sizeof(T) + 16 * dc::kRotScratch2 * sizeof(float2);
  const int64_t cap = static_cast<int64_t>(sm_count()) * 2;
  const int ctas = static_cast<int>(M < cap ? M : cap);
  const int Ki = static_cast<int>(K);
  int r = DC_OK;
  auto go = [&](auto kernel) {
    r = set_smem(kernel, static_cast<int>(smem));
    if (r == DC_OK) kernel<<<ctas, 256, smem, st>>>(src, M, Ki, q, s);
  };
  if (nit2 <= 1) go(dc::rowq_cta_pair_kernel<T, SEG, 1>);
  else go(dc::rowq_cta_pair_kernel<T, SEG, 2>);
  if (r) return r;
  DC_CHECK_LAUNCH("quant_rows launch");
  return DC_OK;
}

template <typename T, bool GROUP, bool SEG>
int launch_rowq_cta(const dc::RowSrc& src, int64_t M, int64_t K, int8_t* q, float* s, cudaStream_t st) {
  if constexpr (GROUP) {
    if (use_rowq_pair()) return launch_rowq_cta_pair<T, SEG>(src, M, K, q, s, st);
  }
  const int nit = static_cast<int>((K / 256 + 15) / 16);
  const size_t smem = 2 * K * sizeof(T) + 16 * dc::kRotScratch * sizeof(float);
  const int64_t cap = static_cast<int64_t>(sm_count()) * 2;
  const int ctas = static_cast<int>(M < cap ? M : cap);
  const int Ki = static_cast<int>(K);
  int r = DC_OK;
  auto go = [&](auto kernel) {
    r = set_smem(kernel, static_cast<int>(smem));
    if (r == DC_OK) kernel<<<ctas, 256, smem, st>>>(src, M, Ki, q, s);
  };
  if (nit <= 2) go(dc::rowq_cta_kernel<T, GROUP, SEG, 2>);
  else if (nit <= 3) go(dc::rowq_cta_kernel<T, GROUP, SEG, 3>);
  else go(dc::rowq_cta_kernel<T, GROUP, SEG, 4>);
  if (r) return r;
  DC_CHECK_LAUNCH("quant_rows launch");
  return DC_OK;
}

template <typename T, bool GROUP, int GELU, bool SEG = false>
int launch_quant_t(const dc::RowSrc& src, int64_t M, int64_t K, int8_t* q, float* s, bool vec, cudaStream_t st) {
  if constexpr (GELU == 0 && sizeof(T) == 2) {
    // Shared-memory streaming kernels where they pay: with the ConvRot rotation (no warp-shuffle
    // butterfly), and for wide rows (no second pass over rows L2 has evicted). Plain rows up to
    // 4096 wide keep the register warp kernel below, which has more rows in flight per SM.
    const int reg = rowq_reg_mode();
    if (vec && K % 256 == 0 && K <= 16384 && reinterpret_cast<uintptr_t>(q) % 16 == 0 &&
        (reg == 2 || (reg == 1 && GROUP)) && (!SEG || src.seg_len >= 256))
      return launch_rowq_reg<T, false, GROUP, SEG>(src, M, K, nullptr, nullptr, q, s, st);
    if (vec && K % 256 == 0 && K <= 16384 && reinterpret_cast<uintptr_t>(q) % 16 == 0 && (GROUP || K > 4096))
      return K <= 4096 ? launch_rowq_warp<T, GROUP, false, SEG>(src, M, K, nullptr, nullptr, q, s, st)
                       : launch_rowq_cta<T, GROUP, SEG>(src, M, K, q, s, st);
  }
  if constexpr (!GROUP && GELU == 0 && sizeof(T) == 2) {
    if (vec && K > 4096) {
      const int64_t ctas64 = (M + 3) / 4;
      const int ctas = static_cast<int>(ctas64 < static_cast<int64_t>(sm_count()) * 48 ? ctas64 : sm_count() * 48);
      dc::quant_rows_stream_kernel<T, SEG><<<ctas, 128, 0, st>>>(src, M, static_cast<int>(K), q, s);
      DC_CHECK_LAUNCH("quant_rows launch");
      return DC_OK;
    }
  }
  if constexpr (!GROUP && GELU == 0 && sizeof(T) == 2) {
    // plain 16-bit rows up to 4096 wide: a CTA per row at full occupancy (unless DC_QUANT_CTA=0)
    const char* env = getenv("DC_QUANT_CTA");
    if (vec && K <= 4096 && (env == nullptr || strcmp(env, "0") != 0)) {
      const int64_t cap = static_cast<int64_t>(sm_count()) * 64;
      const int ctas = static_cast<int>(M < cap ? M : cap);
      const int vpt = static_cast<int>((K / 8 + 127) / 128);
      const int Ki = static_cast<int>(K);
      if (vpt <= 1) dc::quant_rows_cta_kernel<T, 1, SEG><<<ctas, 128, 0, st>>>(src, M, Ki, q, s);
      else if (vpt <= 2) dc::quant_rows_cta_kernel<T, 2, SEG><<<ctas, 128, 0, st>>>(src, M, Ki, q, s);
      else if (vpt <= 3) dc::quant_rows_cta_kernel<T, 3, SEG><<<ctas, 128, 0, st>>>(src, M, Ki, q, s);
      else dc::quant_rows_cta_kernel<T, 4, SEG><<<ctas, 128, 0, st>>>(src, M, Ki, q, s);
      DC_CHECK_LAUNCH("quant_rows launch");
      return DC_OK;
    }
  }
  if (vec && K <= 4096) {
    // warp per row, 4 rows per CTA
    const int64_t ctas64 = (M + 3) / 4;
    const int ctas = static_cast<int>(ctas64 < static_cast<int64_t>(sm_count()) * 32 ? ctas64 : sm_count() * 32);
    const int vpt = static_cast<int>((K / 8 + 31) / 32);
    const int Ki = static_cast<int>(K);
    if (vpt <= 4) dc::quant_rows_warp_kernel<T, 4, GROUP, GELU, SEG><<<ctas, 128, 0, st>>>(src, M, Ki, q, s);
    else if (vpt <= 8) dc::quant_rows_warp_kernel<T, 8, GROUP, GELU, SEG><<<ctas, 128, 0, st>>>(src, M, Ki, q, s);
    else if (vpt <= 12) dc::quant_rows_warp_kernel<T, 12, GROUP, GELU, SEG><<<ctas, 128, 0, st>>>(src, M, Ki, q, s);
    else dc::quant_rows_warp_kernel<T, 16, GROUP, GELU, SEG><<<ctas, 128, 0, st>>>(src, M, Ki, q, s);
  } else if (vec) {
    const int64_t grid64 = M < static_cast<int64_t>(sm_count()) * 16 ? M : static_cast<int64_t>(sm_count()) * 16;
    const int grid = static_cast<int>(grid64);
    const int vpt = static_cast<int>((K / 8 + dc::kQuantThreads - 1) / dc::kQuantThreads);
    const int Ki = static_cast<int>(K);
    if (vpt <= 8) dc::quant_rows_kernel<T, 8, GROUP, GELU, SEG><<<grid, dc::kQuantThreads, 0, st>>>(src, M, Ki, q, s);
    else dc::quant_rows_kernel<T, 16, GROUP, GELU, SEG><<<grid, dc::kQuantThreads, 0, st>>>(src, M, Ki, q, s);
  } else {
    if constexpr (!SEG) {
      const int64_t grid64 = M < static_cast<int64_t>(sm_count()) * 16 ? M : static_cast<int64_t>(sm_count()) * 16;
      dc::quant_rows_scalar_kernel<T, GELU><<<static_cast<int>(grid64), dc::kQuantThreads, 0, st>>>(
          static_cast<const T*>(src.x), M, static_cast<int>(K), src.ldx, q, s, src.full_div);
    } else {
      return fail("segmented quant_rows needs 16-byte aligned segments");
    }
  }
  DC_CHECK_LAUNCH("quant_rows launch");
  return DC_OK;
}

template <typename T>
int launch_quant(const void* x, int64_t M, int64_t K, int64_t ldx, int group, int gelu, int8_t* q, float* s,
                 cudaStream_t st) {
  dc::RowSrc src = dc::plain_rows(x, ldx);
  src.full_div = quant_full_div();
  src.rot_order = dc::rot_order_for_width(K);
  const bool vec = (K % 8 == 0) && (ldx % 8 == 0) && (reinterpret_cast<uintptr_t>(x) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(q) % 8 == 0) && K <= 16384;
  if (group != 0 && !vec) return fail("rotated quantization needs K %% 256 == 0, ldx %% 8 == 0, 16-byte aligned rows");
  if constexpr (std::is_same<T, float>::value) {
    return group ? launch_quant_t<T, true, 0>(src, M, K, q, s, vec, st)
                 : launch_quant_t<T, false, 0>(src, M, K, q, s, vec, st);
  } else {
    switch (gelu) {
      case DC_GELU_ERF:
        return group ? launch_quant_t<T, true, 1>(src, M, K, q, s, vec, st)
                     : launch_quant_t<T, false, 1>(src, M, K, q, s, vec, st);
      case DC_GELU_TANH:
        return group ? launch_quant_t<T, true, 2>(src, M, K, q, s, vec, st)
                     : launch_quant_t<T, false, 2>(src, M, K, q, s, vec, st);
      default:
        return group ? launch_quant_t<T, true, 0>(src, M, K, q, s, vec, st)
                     : launch_quant_t<T, false, 0>(src, M, K, q, s, vec, st);
    }
  }
}

// ------------------------------------------------------------------------------ DiT glue

template <typename T, bool GROUP>
int launch_ln_mod_quant(const void* x, int64_t M, int64_t K, int64_t ldx, const void* shift, const void* scale,
                        int64_t rows_per_mod, int64_t mod_ld, int8_t* q, float* s, cudaStream_t st) {
  const int64_t ctas64 = (M + 3) / 4;
  const int ctas = static_cast<int>(ctas64 < static_cast<int64_t>(sm_count()) * 32 ? ctas64 : sm_count() * 32);
  const int vpt = static_cast<int>((K / 8 + 31) / 32);
  const int Ki = static_cast<int>(K);
  const T* xp = static_cast<const T*>(x);
  const T* sh = static_cast<const T*>(shift);
  const T* sc = static_cast<const T*>(scale);
  if (vpt <= 4) dc::ln_mod_quant_kernel<T, 4, GROUP><<<ctas, 128, 0, st>>>(xp, M, Ki, ldx, sh, sc, rows_per_mod, mod_ld, q, s, quant_full_div());
  else if (vpt <= 8) dc::ln_mod_quant_kernel<T, 8, GROUP><<<ctas, 128, 0, st>>>(xp, M, Ki, ldx, sh, sc, rows_per_mod, mod_ld, q, s, quant_full_div());
  else if (vpt <= 12) dc::ln_mod_quant_kernel<T, 12, GROUP><<<ctas, 128, 0, st>>>(xp, M, Ki, ldx, sh, sc, rows_per_mod, mod_ld, q, s, quant_full_div());
  else dc::ln_mod_quant_kernel<T, 16, GROUP><<<ctas, 128, 0, st>>>(xp, M, Ki, ldx, sh, sc, rows_per_mod, mod_ld, q, s, quant_full_div());
  DC_CHECK_LAUNCH("ln_mod_quant launch");
  return DC_OK;
}

// ------------------------------------------------------------------------------ GEMM

// Epilogue options beyond rescale / bias / GELU.
struct GemmEpi {
  const void* gate = nullptr;       // with residual: out = dtype(residual + dtype(gate * y))
  const void* residual = nullptr;
  int64_t ldr = 0;
  int64_t col_block = 0;            // > 0: column-block output layout
  int64_t block_stride = 0;
};

// Pair tiles (256 x 256 over a cluster of two CTAs, see gemm.cuh): the default for GEMMs of at
// least 512 rows, where with 256-byte k-blocks they measured faster on a B200 than the one-CTA
// tile with bit-identical results (config 1: 40.0 vs 41.8 us; FLUX qkv 100.0 vs 108.1; linear2
// 145.2 vs 161.7; the GELU up-projection 156.9 vs 166.4). Environment DC_GEMM_PAIR = "0" turns
// them off, "1" uses them wherever M > 128.
bool use_pair_gemm(int64_t M, int gelu) {
  (void)gelu;
  const char* env = getenv("DC_GEMM_PAIR");
  if (env != nullptr && strcmp(env, "0") == 0) return false;
  if (env != nullptr && strcmp(env, "1") == 0) return M > dc::kGemmBM;
  return M >= 512;
}

// Largest number of two-CTA clusters of `kernel` resident at once on the current device.
template <typename Kern>
int max_pair_clusters(Kern kernel, int smem_bytes, int* clusters) {
  static std::atomic<int> cache[64];                 // per device ordinal; 0 = not computed
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && cache[dev].load() > 0) { *clusters = cache[dev].load(); return DC_OK; }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2; attr[0].val.clusterDim.y = 1; attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(2 * static_cast<unsigned>(sm_count()));
  cfg.blockDim = dim3(dc::kGemmThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem_bytes);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  cudaError_t e = cudaOccupancyMaxActiveClusters(&n, kernel, &cfg);
  if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveClusters");
  if (n <= 0) return fail("gemm: no two-CTA cluster of the pair kernel fits on this device");
  if (dev >= 0 && dev < 64) cache[dev].store(n);
  *clusters = n;
  return DC_OK;
}

template <int BN, int OUT, bool HAS_BIAS, int GELU, bool GATED, bool PAIR = false>
int launch_gemm(const int8_t* q, int64_t ldq, const int8_t* w, int64_t ldw, const float* sx, const float* sw,
                const void* bias, void* out, int64_t ldo, int64_t M, int64_t N, int64_t K, const GemmEpi& epi,
                cudaStream_t st) {
  // Pair and 128-wide tiles stage 256-byte k-blocks (two swizzle atoms) in 3 stages of 64 KB; the
  // one-CTA 256-wide tile 128-byte k-blocks in 4 stages of 48 KB. Measured on a B200: the 256-byte
  // k-blocks took config 1 from 41.1 to 40.0 us, FLUX's qkv from 104.3 to 100.0 us and linear2
  // from 155.4 to 145.2 us (pair tiles).
  constexpr int KATOMS = (PAIR || BN == 128) ? 2 : 1;
  constexpr int STAGES = KATOMS == 2 ? 3 : 4;
  constexpr int kTileM = PAIR ? 2 * dc::kGemmBM : dc::kGemmBM;
  constexpr int kBoxB = PAIR ? BN / 2 : BN;          // B rows one CTA loads per k-block
  using S = dc::GemmSmem<kBoxB, STAGES, KATOMS>;
  CUtensorMap ta, tb;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
    const uint64_t strides[1] = {static_cast<uint64_t>(ldq)};
    const uint32_t box[2] = {dc::kGemmAtom, dc::kGemmBM};
    int r = make_map(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, q, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (r) return r;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(N)};
    const uint64_t strides[1] = {static_cast<uint64_t>(ldw)};
    const uint32_t box[2] = {dc::kGemmAtom, static_cast<uint32_t>(kBoxB)};
    int r = make_map(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, w, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (r) return r;
  }
  dc::GemmParams p;
  p.M = static_cast<int>(M); p.N = static_cast<int>(N); p.K = static_cast<int>(K);
  p.tiles_m = static_cast<int>((M + kTileM - 1) / kTileM);
  p.tiles_n = static_cast<int>((N + BN - 1) / BN);
  p.num_tiles = p.tiles_m * p.tiles_n;
  p.num_kb = static_cast<int>((K + S::kBK - 1) / S::kBK);
  p.sx = sx; p.sw = sw; p.bias = bias; p.out = out; p.ldo = ldo;
  p.gate = epi.gate; p.residual = epi.residual; p.ldr = epi.ldr;
  p.col_block = epi.col_block; p.block_stride = epi.block_stride;
  // Vector (16-byte) stores and residual loads only where every such address is 16-byte aligned:
  // the tile's columns start at multiples of 32 elements, so the base and the row strides decide.
  const int64_t row_elems = OUT == dc::kOutI32 ? 4 : 8;          // elements per 16 bytes
  p.out_vec = reinterpret_cast<uintptr_t>(out) % 16 == 0 && ldo % row_elems == 0 &&
              epi.block_stride % row_elems == 0;
  p.res_vec = epi.residual != nullptr && reinterpret_cast<uintptr_t>(epi.residual) % 16 == 0 &&
              epi.ldr % 8 == 0;
  auto kernel = dc::gemm_w8a8_kernel<BN, STAGES, OUT, HAS_BIAS, GELU, GATED, PAIR, KATOMS>;
  int r = set_smem(kernel, S::kDynamic);
  if (r) return r;
  if constexpr (PAIR) {
    int clusters = 0;
    if ((r = max_pair_clusters(kernel, S::kDynamic, &clusters))) return r;
    const int pairs = p.num_tiles < clusters ? p.num_tiles : clusters;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2; attr[0].val.clusterDim.y = 1; attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * static_cast<unsigned>(pairs));
    cfg.blockDim = dim3(dc::kGemmThreads);
    cfg.dynamicSmemBytes = static_cast<size_t>(S::kDynamic);
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, ta, tb, p);
    if (e != cudaSuccess) return cuda_fail(e, "gemm_w8a8 pair launch");
  } else {
    const int grid = p.num_tiles < sm_count() ? p.num_tiles : sm_count();
    kernel<<<grid, dc::kGemmThreads, S::kDynamic, st>>>(ta, tb, p);
  }
  DC_CHECK_LAUNCH("gemm_w8a8 launch");
  return DC_OK;
}

template <int BN, int OUT, bool PAIR>
int dispatch_gemm_epilogue(const int8_t* q, int64_t ldq, const int8_t* w, int64_t ldw, const float* sx,
                           const float* sw, const void* bias, void* out, int64_t ldo, int64_t M, int64_t N,
                           int64_t K, int gelu, const GemmEpi& epi, cudaStream_t st) {
  if constexpr (OUT == dc::kOutI32) {
    return launch_gemm<BN, OUT, false, 0, false, PAIR>(q, ldq, w, ldw, sx, sw, nullptr, out, ldo, M, N, K, epi, st);
  } else {
    const bool b = bias != nullptr;
    if (epi.residual != nullptr) {
      return b ? launch_gemm<BN, OUT, true, 0, true, PAIR>(q, ldq, w, ldw, sx, sw, bias, out, ldo, M, N, K, epi, st)
               : launch_gemm<BN, OUT, false, 0, true, PAIR>(q, ldq, w, ldw, sx, sw, bias, out, ldo, M, N, K, epi, st);
    }
    switch (gelu) {
      case DC_GELU_NONE:
        return b ? launch_gemm<BN, OUT, true, 0, false, PAIR>(q, ldq, w, ldw, sx, sw, bias, out, ldo, M, N, K, epi, st)
                 : launch_gemm<BN, OUT, false, 0, false, PAIR>(q, ldq, w, ldw, sx, sw, bias, out, ldo, M, N, K, epi, st);
      case DC_GELU_ERF:
        return b ? launch_gemm<BN, OUT, true, 1, false, PAIR>(q, ldq, w, ldw, sx, sw, bias, out, ldo, M, N, K, epi, st)
                 : launch_gemm<BN, OUT, false, 1, false, PAIR>(q, ldq, w, ldw, sx, sw, bias, out, ldo, M, N, K, epi, st);
      default:
        return b ? launch_gemm<BN, OUT, true, 2, false, PAIR>(q, ldq, w, ldw, sx, sw, bias, out, ldo, M, N, K, epi, st)
                 : launch_gemm<BN, OUT, false, 2, false, PAIR>(q, ldq, w, ldw, sx, sw, bias, out, ldo, M, N, K, epi, st);
    }
  }
}

// 128 x 256 tiles on one SM, or 256 x 256 tiles on a CTA pair.
template <int OUT>
int dispatch_gemm_wide(const int8_t* q, int64_t ldq, const int8_t* w, int64_t ldw, const float* sx,
                       const float* sw, const void* bias, void* out, int64_t ldo, int64_t M, int64_t N,
                       int64_t K, int gelu, const GemmEpi& epi, cudaStream_t st) {
  if (use_pair_gemm(M, gelu))
    return dispatch_gemm_epilogue<256, OUT, true>(q, ldq, w, ldw, sx, sw, bias, out, ldo, M, N, K, gelu, epi, st);
  return dispatch_gemm_epilogue<256, OUT, false>(q, ldq, w, ldw, sx, sw, bias, out, ldo, M, N, K, gelu, epi, st);
}

int gemm_checked(const int8_t* q, int64_t ldq, const int8_t* w, int64_t ldw, const float* sx, const float* sw,
                 const void* bias, void* out, int64_t ldo, int out_dtype, int64_t M, int64_t N, int64_t K, int gelu,
                 const GemmEpi& epi, cudaStream_t st) {
  if (M < 0 || N <= 0 || K <= 0) return fail("gemm: bad shape M=%lld N=%lld K=%lld", (long long)M, (long long)N, (long long)K);
  if (M == 0) return DC_OK;
  if (K % 16) return fail("gemm: K=%lld must be a multiple of 16 (TMA row pitch)", (long long)K);
  if (ldq % 16 || ldw % 16) return fail("gemm: ldq/ldw must be multiples of 16 bytes");
  if (ldq < K || ldw < K) return fail("gemm: leading dimension smaller than the row");
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return fail("gemm: dimension above 2^31");
  if (gelu < 0 || gelu > 2) return fail("unknown gelu mode %d", gelu);
  if (q == nullptr || w == nullptr || out == nullptr) return fail("gemm: null operand or output");
  if (out_dtype != DC_DTYPE_I32 && (sx == nullptr || sw == nullptr)) return fail("gemm: scales are required");
  if (out_dtype == DC_DTYPE_I32 && (bias != nullptr || gelu)) return fail("gemm: int32 output takes no bias or gelu");
  if ((epi.gate == nullptr) != (epi.residual == nullptr)) return fail("gemm: gate and residual go together");
  {
    const uintptr_t elem = out_dtype == DC_DTYPE_I32 ? 4 : 2;      // element-aligned pointers
    if (reinterpret_cast<uintptr_t>(out) % elem || reinterpret_cast<uintptr_t>(bias) % 2 ||
        reinterpret_cast<uintptr_t>(epi.gate) % 2 || reinterpret_cast<uintptr_t>(epi.residual) % 2 ||
        reinterpret_cast<uintptr_t>(sx) % 4 || reinterpret_cast<uintptr_t>(sw) % 4)
      return fail("gemm: out, bias, gate, residual and scales must be aligned to their element size");
  }
  if (epi.residual != nullptr) {
    if (out_dtype == DC_DTYPE_I32) return fail("gemm: a gated residual needs a 16-bit output");
    if (gelu) return fail("gemm: a gated residual takes no gelu");
    if (epi.ldr < N) return fail("gemm: residual leading dimension smaller than the row");
  }
  // Wide (128 x 256) tiles unless the column blocks are not a multiple of them, or unless 128 x 128
  // tiles fill the SMs in fewer tile-times: with few 128-row blocks (a sequence-parallel rank's rows,
  // FLUX's 512 text rows) the wide grid can leave most SMs idle. Cost = waves x tile width; the wide
  // tile wins ties (it re-reads each activation block half as often).
  bool wide = N > 128;
  if (wide) {
    const int64_t tm = (M + dc::kGemmBM - 1) / dc::kGemmBM, sms = sm_count();
    const int64_t cost_wide = (tm * ((N + 255) / 256) + sms - 1) / sms * 256;
    const int64_t cost_narrow = (tm * ((N + 127) / 128) + sms - 1) / sms * 128;
    if (cost_narrow * 100 <= cost_wide * 85) wide = false;
  }
  if (epi.col_block > 0) {
    if (epi.col_block % 128 || epi.block_stride % 8) return fail("gemm: col_block must be a multiple of 128 and block_stride of 8");
    if (ldo < epi.col_block) return fail("gemm: ldo smaller than col_block");
    if (epi.col_block % 256) wide = false;
  } else if (ldo < N) {
    return fail("gemm: leading dimension smaller than the row");
  }
  if (int r = check_sm100()) return r;
  switch (out_dtype) {
    case DC_DTYPE_BF16:
      return wide ? dispatch_gemm_wide<dc::kOutBF16>(q, ldq, w, ldw, sx, sw, bias, out, ldo, M, N, K, gelu, epi, st)
                  : dispatch_gemm_epilogue<128, dc::kOutBF16, false>(q, ldq, w, ldw, sx, sw, bias, out, ldo, M, N, K, gelu, epi, st);
    case DC_DTYPE_F16:
      return wide ? dispatch_gemm_wide<dc::kOutF16>(q, ldq, w, ldw, sx, sw, bias, out, ldo, M, N, K, gelu, epi, st)
                  : dispatch_gemm_epilogue<128, dc::kOutF16, false>(q, ldq, w, ldw, sx, sw, bias, out, ldo, M, N, K, gelu, epi, st);
    case DC_DTYPE_I32:
      return wide ? dispatch_gemm_wide<dc::kOutI32>(q, ldq, w, ldw, sx, sw, nullptr, out, ldo, M, N, K, 0, epi, st)
                  : dispatch_gemm_epilogue<128, dc::kOutI32, false>(q, ldq, w, ldw, sx, sw, nullptr, out, ldo, M, N, K, 0, epi, st);
    default: return fail("gemm: unsupported output dtype %d", out_dtype);
  }
}

// ------------------------------------------------------------------------------ attention

struct AttnLayout {
  int64_t Lq_pad, Lk_pad, nwin;
  size_t q_codes, k_codes, q_scale, k_scale, kpart, ksum, total;
};

AttnLayout attn_layout(int64_t B, int64_t H, int64_t Lq, int64_t Lk, int64_t D, int mode) {
  AttnLayout a;
  a.Lq_pad = round_up(Lq, dc::kAttnRows);
  a.Lk_pad = round_up(Lk, dc::kAttnBN);
  a.nwin = (Lk + dc::kStatWin - 1) / dc::kStatWin;
  const int64_t BH = B * H;
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off += static_cast<size_t>(round_up(static_cast<int64_t>(bytes), 256)); return o; };
  a.q_codes = take(static_cast<size_t>(BH * a.Lq_pad * D));
  a.k_codes = take(static_cast<size_t>(BH * a.Lk_pad * D));
  a.q_scale = take(static_cast<size_t>(BH * a.Lq_pad) * 4);
  a.k_scale = take(static_cast<size_t>(BH * (a.Lk_pad / dc::kAttnKBlk)) * 4);
  if (mode == dc::kModeRef) {
    a.kpart = take(static_cast<size_t>(BH * a.nwin * D) * 4);
    a.ksum = take(static_cast<size_t>(BH * D) * 4);
  } else {
    a.kpart = a.ksum = 0;
  }
  a.total = off;
  return a;
}

int check_attn_args(int dtype, int64_t B, int64_t H, int64_t Lq, int64_t Lk, int64_t D, int mode) {
  if (dtype != DC_DTYPE_F16 && dtype != DC_DTYPE_BF16) return fail("attention dtype must be fp16 or bf16");
  if (D != 64 && D != 128) return fail("attention head dim must be 64 or 128 (got %lld)", (long long)D);
  if (mode != DC_ATTN_MODE_REF && mode != DC_ATTN_MODE_BLOCK64) return fail("unknown attention quant mode %d", mode);
  if (B <= 0 || H <= 0 || Lq <= 0 || Lk <= 0) return fail("empty attention input");
  if (B > 65535 || H > 65535) return fail("B and H must be < 65536");
  if (Lq > (1 << 24) || Lk > (1 << 24)) return fail("sequence length above 2^24");
  return DC_OK;
}

int check_strides(const void* ptr, const int64_t* s, const char* name) {
  if (ptr == nullptr || s == nullptr) return fail("%s or its strides is null", name);
  if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0) return fail("%s must be 16-byte aligned", name);
  for (int i = 0; i < 3; ++i)
    if (s[i] % 8 != 0 || s[i] < 0) return fail("%s strides must be non-negative multiples of 8 elements", name);
  return DC_OK;
}

// do_q = false: the Q codes and scales are already in the workspace (dc_qk_norm_rope_q8).
template <typename T, int D>
int attn_prep(const void* q, const void* k, int64_t B, int64_t H, int64_t Lq, int64_t Lk, const int64_t* qs,
              const int64_t* ks, int mode, uint8_t* ws, const AttnLayout& a, cudaStream_t st, bool do_q = true) {
  int8_t* q_codes = reinterpret_cast<int8_t*>(ws + a.q_codes);
  int8_t* k_codes = reinterpret_cast<int8_t*>(ws + a.k_codes);
  float* q_scale = reinterpret_cast<float*>(ws + a.q_scale);
  float* k_scale = reinterpret_cast<float*>(ws + a.k_scale);
  const T* qp = static_cast<const T*>(q);
  const T* kp = static_cast<const T*>(k);
  const int Hi = static_cast<int>(H);
  if (mode == dc::kModeRef) {
    float* kpart = reinterpret_cast<float*>(ws + a.kpart);
    float* ksum = reinterpret_cast<float*>(ws + a.ksum);
    dc::k_stats_kernel<T, D><<<dim3(static_cast<unsigned>(a.nwin), Hi, static_cast<unsigned>(B)), 16 * (D / 8), 0, st>>>(
        kp, kpart, static_cast<int>(Lk), Hi, ks[0], ks[1], ks[2]);
    dc::k_sum_kernel<D><<<static_cast<unsigned>(B * H), D, 0, st>>>(kpart, ksum, static_cast<int>(a.nwin));
    dc::block_quant_kernel<T, D><<<dim3(static_cast<unsigned>(a.Lk_pad / dc::kAttnKBlk), Hi, static_cast<unsigned>(B)), 256, 0, st>>>(
        kp, ksum, k_codes, k_scale, nullptr, static_cast<int>(Lk), Hi, static_cast<int>(a.Lk_pad), ks[0], ks[1], ks[2]);
    constexpr int rows_per_cta = 256 / (D / 8);
    if (do_q) dc::q_token_quant_kernel<T, D><<<dim3(static_cast<unsigned>((a.Lq_pad + rows_per_cta - 1) / rows_per_cta), Hi,
                                          static_cast<unsigned>(B)), 256, 0, st>>>(
        qp, q_codes, q_scale, static_cast<int>(Lq), Hi, static_cast<int>(a.Lq_pad), qs[0], qs[1], qs[2]);
  } else {
    dc::block_quant_kernel<T, D><<<dim3(static_cast<unsigned>(a.Lk_pad / dc::kAttnKBlk), Hi, static_cast<unsigned>(B)), 256, 0, st>>>(
        kp, nullptr, k_codes, k_scale, nullptr, static_cast<int>(Lk), Hi, static_cast<int>(a.Lk_pad), ks[0], ks[1], ks[2]);
    // Q per 64-row block: only the per-row copy of the block scale is kept (the main kernel
    // reads one scale per query row in both modes).
    if (do_q) dc::block_quant_kernel<T, D><<<dim3(static_cast<unsigned>(a.Lq_pad / dc::kAttnKBlk), Hi, static_cast<unsigned>(B)), 256, 0, st>>>(
        qp, nullptr, q_codes, nullptr, q_scale, static_cast<int>(Lq), Hi, static_cast<int>(a.Lq_pad), qs[0], qs[1],
        qs[2]);
  }
  DC_CHECK_LAUNCH("attention prep launch");
  return DC_OK;
}

// Which main kernel: both run one CTA per SM (each holds all 512 TMEM columns). The two-tile
// kernel (256 query rows per CTA) does more work per CTA-time; the single-tile kernel (128 rows,
// S double-buffered) takes 0.61 of its time per CTA (measured on B200 at B=1, H=24, L=4608:
// 49 vs 81 us per wave) and so wins when the two-tile grid ends in a poorly filled wave (few
// heads per GPU, as with a sequence-parallel split). Environment DC_ATTN_KERNEL = "two_tile" or
// "single_tile" pins one (tests use it to cover both).
bool use_single_tile_kernel(int64_t ctas_two_tile, int64_t ctas_single_tile) {
  const char* env = getenv("DC_ATTN_KERNEL");
  if (env != nullptr && strcmp(env, "two_tile") == 0) return false;
  if (env != nullptr && strcmp(env, "single_tile") == 0) return true;
  const int64_t sms = sm_count();
  const double waves_two = static_cast<double>((ctas_two_tile + sms - 1) / sms);
  const double waves_single = static_cast<double>((ctas_single_tile + sms - 1) / sms);
  return 0.61 * waves_single < waves_two;
}

template <typename T, int D>
int attn_main(const void* v, int64_t B, int64_t H, int64_t Lq, int64_t Lk, const int64_t* vs, float sm_scale,
              void* o, const int64_t* os, uint8_t* ws, const AttnLayout& a, cudaStream_t st) {
  constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
  using SM = dc::AttnSmem<D>;
  CUtensorMap tq, tk, tv;
  const CUtensorMapSwizzle qk_swz = D == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(D), static_cast<uint64_t>(B * H * a.Lq_pad)};
    const uint64_t strides[1] = {static_cast<uint64_t>(D)};
    const uint32_t box[2] = {static_cast<uint32_t>(D), dc::kAttnBM};
    int r = make_map(&tq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, ws + a.q_codes, dims, strides, box, qk_swz);
    if (r) return r;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(D), static_cast<uint64_t>(B * H * a.Lk_pad)};
    const uint64_t strides[1] = {static_cast<uint64_t>(D)};
    const uint32_t box[2] = {static_cast<uint32_t>(D), dc::kAttnBN};
    int r = make_map(&tk, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, ws + a.k_codes, dims, strides, box, qk_swz);
    if (r) return r;
  }
  {
    const uint64_t dims[4] = {static_cast<uint64_t>(D), static_cast<uint64_t>(Lk), static_cast<uint64_t>(H),
                              static_cast<uint64_t>(B)};
    const uint64_t strides[3] = {static_cast<uint64_t>(vs[1]) * 2, static_cast<uint64_t>(vs[2]) * 2,
                                 static_cast<uint64_t>(vs[0]) * 2};
    const uint32_t box[4] = {64, dc::kAttnBN, 1, 1};
    int r = make_map(&tv, BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, v, dims,
                     strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (r) return r;
  }
  dc::AttnParams p;
  p.H = static_cast<int>(H); p.Lq = static_cast<int>(Lq); p.Lk = static_cast<int>(Lk);
  p.Lq_pad = static_cast<int>(a.Lq_pad); p.Lk_pad = static_cast<int>(a.Lk_pad);
  p.n_ktiles = static_cast<int>(a.Lk_pad / dc::kAttnBN);
  p.scale_log2 = sm_scale * 1.4426950408889634f;
  p.q_scale = reinterpret_cast<const float*>(ws + a.q_scale);
  p.k_scale = reinterpret_cast<const float*>(ws + a.k_scale);
  p.o = o; p.o_sb = os[0]; p.o_sl = os[1]; p.o_sh = os[2];
  if (use_single_tile_kernel(B * H * (a.Lq_pad / dc::kAttnRows), B * H * (a.Lq_pad / dc::kDbRows))) {
    using SD = dc::AttnDbSmem<D>;
    auto kernel = dc::attn_db_kernel<D, BF16>;
    int r = set_smem(kernel, SD::kDynamic);
    if (r) return r;
    dim3 grid(static_cast<unsigned>(a.Lq_pad / dc::kDbRows), static_cast<unsigned>(H), static_cast<unsigned>(B));
    kernel<<<grid, dc::kAttnThreads, SD::kDynamic, st>>>(tq, tk, tv, p);
  } else {
    auto kernel = dc::attn_int8_kernel<D, BF16, false>;
    int r = set_smem(kernel, SM::kDynamic);
    if (r) return r;
    dim3 grid(static_cast<unsigned>(a.Lq_pad / dc::kAttnRows), static_cast<unsigned>(H), static_cast<unsigned>(B));
    kernel<<<grid, dc::kAttnThreads, SM::kDynamic, st>>>(tq, tk, tv, p);
  }
  DC_CHECK_LAUNCH("attention launch");
  return DC_OK;
}

// Key ranges of the split attention: tiles_per_split = ceil(n / nsplit) key tiles each, and as many
// ranges as that takes (every range non-empty).
inline void split_ranges(int64_t n_ktiles, int nsplit, int* tiles_per_split, int* ranges) {
  const int64_t tps = (n_ktiles + nsplit - 1) / nsplit;
  *tiles_per_split = static_cast<int>(tps);
  *ranges = static_cast<int>((n_ktiles + tps - 1) / tps);
}

inline size_t split_partial_bytes(int64_t BH, int64_t Lq_pad, int64_t D, int nsplit) {
  return static_cast<size_t>(nsplit) * static_cast<size_t>(BH * Lq_pad) * (static_cast<size_t>(D) * 4 + 8);
}

// attn_main with the keys divided into ranges (attn_int8_kernel<..., SPLIT = true>, two Q tiles per
// CTA, one CTA per (Q pair, key range)) and the ranges merged by attn_split_combine_kernel. The
// tensor maps are attn_main's.
template <typename T, int D>
int attn_main_split(const void* v, int64_t B, int64_t H, int64_t Lq, int64_t Lk, const int64_t* vs, float sm_scale,
                    void* o, const int64_t* os, uint8_t* ws, const AttnLayout& a, int nsplit, void* partials,
                    cudaStream_t st) {
  constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
  using SM = dc::AttnSmem<D>;
  CUtensorMap tq, tk, tv;
  const CUtensorMapSwizzle qk_swz = D == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(D), static_cast<uint64_t>(B * H * a.Lq_pad)};
    const uint64_t strides[1] = {static_cast<uint64_t>(D)};
    const uint32_t box[2] = {static_cast<uint32_t>(D), dc::kAttnBM};
    int r = make_map(&tq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, ws + a.q_codes, dims, strides, box, qk_swz);
    if (r) return r;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(D), static_cast<uint64_t>(B * H * a.Lk_pad)};
    const uint64_t strides[1] = {static_cast<uint64_t>(D)};
    const uint32_t box[2] = {static_cast<uint32_t>(D), dc::kAttnBN};
    int r = make_map(&tk, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, ws + a.k_codes, dims, strides, box, qk_swz);
    if (r) return r;
  }
  {
    const uint64_t dims[4] = {static_cast<uint64_t>(D), static_cast<uint64_t>(Lk), static_cast<uint64_t>(H),
                              static_cast<uint64_t>(B)};
    const uint64_t strides[3] = {static_cast<uint64_t>(vs[1]) * 2, static_cast<uint64_t>(vs[2]) * 2,
                                 static_cast<uint64_t>(vs[0]) * 2};
    const uint32_t box[4] = {64, dc::kAttnBN, 1, 1};
    int r = make_map(&tv, BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, v, dims,
                     strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (r) return r;
  }
  dc::AttnParams p;
  p.H = static_cast<int>(H); p.Lq = static_cast<int>(Lq); p.Lk = static_cast<int>(Lk);
  p.Lq_pad = static_cast<int>(a.Lq_pad); p.Lk_pad = static_cast<int>(a.Lk_pad);
  p.n_ktiles = static_cast<int>(a.Lk_pad / dc::kAttnBN);
  p.scale_log2 = sm_scale * 1.4426950408889634f;
  p.q_scale = reinterpret_cast<const float*>(ws + a.q_scale);
  p.k_scale = reinterpret_cast<const float*>(ws + a.k_scale);
  p.o = o; p.o_sb = os[0]; p.o_sl = os[1]; p.o_sh = os[2];
  int ranges = 1;
  split_ranges(p.n_ktiles, nsplit, &p.tiles_per_split, &ranges);
  p.nsplit = ranges;
  p.BH = static_cast<int>(B * H);
  p.part_o = static_cast<float*>(partials);
  p.part_ml = reinterpret_cast<float2*>(static_cast<uint8_t*>(partials) +
                                        static_cast<size_t>(ranges) * static_cast<size_t>(B * H * a.Lq_pad) * D * 4);
  auto kernel = dc::attn_int8_kernel<D, BF16, true>;
  int r = set_smem(kernel, SM::kDynamic);
  if (r) return r;
  dim3 grid(static_cast<unsigned>(a.Lq_pad / dc::kAttnRows * ranges), static_cast<unsigned>(H), static_cast<unsigned>(B));
  kernel<<<grid, dc::kAttnThreads, SM::kDynamic, st>>>(tq, tk, tv, p);
  DC_CHECK_LAUNCH("split attention launch");
  const int64_t rows = B * H * Lq;
  const unsigned blocks = static_cast<unsigned>((rows + 7) / 8);          // 8 warps (rows) per block
  dc::attn_split_combine_kernel<D, BF16><<<blocks, 256, 0, st>>>(p.part_o, p.part_ml, ranges, p.BH, p.H, p.Lq,
                                                                 p.Lq_pad, o, os[0], os[1], os[2]);
  DC_CHECK_LAUNCH("split attention combine launch");
  return DC_OK;
}

__global__ void selftest_wait_kernel(long long limit, int* status) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    dc::mbar_init(&bar, 1);
    abort_flag = 0;
    dc::fence_barrier_init();
  }
  __syncthreads();
  // Nothing arrives on `bar`: the bounded wait must give up and report it.
  const bool ok = dc::mbar_wait(&bar, 0, &abort_flag, limit);
  if (threadIdx.x == 0) {
    *status = ok ? 0 : 1;
    if (!ok) atomicCAS(&dc::g_device_error, static_cast<unsigned int>(dc::kErrWaitTimeout),
                       static_cast<unsigned int>(dc::kErrSelfTest));
  }
}

__global__ void selftest_exp2_kernel(const float* __restrict__ x, float* __restrict__ poly, float* __restrict__ ref,
                                     int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (2 * i + 1 < n) {
    const float2 p = dc::exp2_poly2(make_float2(x[2 * i], x[2 * i + 1]));
    poly[2 * i] = p.x;
    poly[2 * i + 1] = p.y;
    ref[2 * i] = exp2f(x[2 * i]);
    ref[2 * i + 1] = exp2f(x[2 * i + 1]);
  }
}

}  // namespace

extern "C" {

int dc_version(void) { return DC_ABI_VERSION; }

int dc_set_quant_division(int mode) {
  if (mode != DC_QDIV_IEEE && mode != DC_QDIV_FULL) return fail("unknown quantizer division mode %d", mode);
  g_quant_div.store(mode, std::memory_order_relaxed);
  return DC_OK;
}

int dc_quant_division(void) { return g_quant_div.load(std::memory_order_relaxed); }

const char* dc_last_error(void) { return g_err; }

int dc_device_error(unsigned int* code, int clear) {
  unsigned int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, dc::g_device_error, sizeof(v));
  if (e != cudaSuccess) return cuda_fail(e, "reading the device error word");
  if (clear) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(dc::g_device_error, &zero, sizeof(zero));
    if (e != cudaSuccess) return cuda_fail(e, "clearing the device error word");
  }
  if (code) *code = v;
  return DC_OK;
}

int dc_quant_rows(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, int group, int gelu, int8_t* q,
                  float* s, void* stream) {
  if (M < 0 || K <= 0) return fail("quant_rows: bad shape M=%lld K=%lld", (long long)M, (long long)K);
  if (M == 0) return DC_OK;
  if (group != 0 && group != 256) return fail("ConvRot group must be 0 or 256 (got %d)", group);
  if (group && K % 256) return fail("K=%lld is not a multiple of the ConvRot group 256", (long long)K);
  if (ldx < K) return fail("ldx < K");
  if (gelu < 0 || gelu > 2) return fail("unknown gelu mode %d", gelu);
  if (x == nullptr || q == nullptr || s == nullptr) return fail("quant_rows: null pointer");
  if (reinterpret_cast<uintptr_t>(x) % (x_dtype == DC_DTYPE_F32 ? 4 : 2) || reinterpret_cast<uintptr_t>(s) % 4)
    return fail("quant_rows: x and s must be aligned to their element size");
  if (int r = check_sm100()) return r;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (x_dtype) {
    case DC_DTYPE_BF16: return launch_quant<__nv_bfloat16>(x, M, K, ldx, group, gelu, q, s, st);
    case DC_DTYPE_F16: return launch_quant<__half>(x, M, K, ldx, group, gelu, q, s, st);
    case DC_DTYPE_F32:
      if (gelu) return fail("gelu needs a 16-bit input dtype");
      return launch_quant<float>(x, M, K, ldx, group, 0, q, s, st);
    default: return fail("quant_rows: unsupported dtype %d", x_dtype);
  }
}

int dc_gemm_w8a8(const int8_t* q, int64_t ldq, const int8_t* w, int64_t ldw, const float* sx, const float* sw,
                 const void* bias, void* out, int64_t ldo, int out_dtype, int64_t M, int64_t N, int64_t K,
                 int gelu, void* stream) {
  return gemm_checked(q, ldq, w, ldw, sx, sw, bias, out, ldo, out_dtype, M, N, K, gelu, GemmEpi(),
                      static_cast<cudaStream_t>(stream));
}

int dc_gemm_w8a8_ex(const int8_t* q, int64_t ldq, const int8_t* w, int64_t ldw, const float* sx, const float* sw,
                    const void* bias, int gelu, const void* gate, const void* residual, int64_t ldr, void* out,
                    int64_t ldo, int64_t col_block, int64_t block_stride, int out_dtype, int64_t M, int64_t N,
                    int64_t K, void* stream) {
  GemmEpi epi;
  epi.gate = gate; epi.residual = residual; epi.ldr = ldr;
  epi.col_block = col_block; epi.block_stride = block_stride;
  if (col_block < 0 || (col_block == 0 && block_stride != 0)) return fail("gemm: bad column-block layout");
  return gemm_checked(q, ldq, w, ldw, sx, sw, bias, out, ldo, out_dtype, M, N, K, gelu, epi,
                      static_cast<cudaStream_t>(stream));
}

int dc_quant_rows_seg(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, int64_t seg_len,
                      int64_t seg_stride, int64_t k1, const void* x2, int64_t ldx2, int group, int8_t* q, float* s,
                      void* stream) {
  if (M < 0 || K <= 0) return fail("quant_rows_seg: bad shape");
  if (M == 0) return DC_OK;
  if (x == nullptr || q == nullptr || s == nullptr) return fail("quant_rows_seg: null pointer");
  if (reinterpret_cast<uintptr_t>(s) % 4) return fail("quant_rows_seg: s must be 4-byte aligned");
  if (group != 0 && group != 256) return fail("ConvRot group must be 0 or 256 (got %d)", group);
  if (group && K % 256) return fail("K=%lld is not a multiple of the ConvRot group 256", (long long)K);
  if (K % 8 || K > 16384) return fail("quant_rows_seg: K must be a multiple of 8 and at most 16384");
  if (seg_len <= 0 || seg_len % 8 || k1 <= 0 || k1 > K || k1 % seg_len)
    return fail("quant_rows_seg: seg_len must be a positive multiple of 8 dividing k1, 0 < k1 <= K");
  if (seg_stride % 8 || ldx % 8 || ldx < seg_len) return fail("quant_rows_seg: strides must be multiples of 8 elements");
  if (k1 < K && (x2 == nullptr || ldx2 % 8 || ldx2 < K - k1 || reinterpret_cast<uintptr_t>(x2) % 16))
    return fail("quant_rows_seg: the second operand needs a 16-byte aligned base and ldx2 >= K - k1, a multiple of 8");
  if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(q) % 8)
    return fail("quant_rows_seg: x must be 16-byte and q 8-byte aligned");
  if (x_dtype != DC_DTYPE_BF16 && x_dtype != DC_DTYPE_F16) return fail("quant_rows_seg: dtype must be fp16 or bf16");
  if (int r = check_sm100()) return r;
  dc::RowSrc src;
  src.x = x; src.ldx = ldx; src.seg_len = static_cast<int>(seg_len); src.seg_stride = seg_stride;
  src.k1 = static_cast<int>(k1); src.x2 = x2; src.ldx2 = ldx2; src.full_div = quant_full_div();
  src.rot_order = dc::rot_order_for_width(K);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (x_dtype == DC_DTYPE_BF16)
    return group ? launch_quant_t<__nv_bfloat16, true, 0, true>(src, M, K, q, s, true, st)
                 : launch_quant_t<__nv_bfloat16, false, 0, true>(src, M, K, q, s, true, st);
  return group ? launch_quant_t<__half, true, 0, true>(src, M, K, q, s, true, st)
               : launch_quant_t<__half, false, 0, true>(src, M, K, q, s, true, st);
}

int dc_ln_mod_quant(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, const void* shift,
                    const void* scale, int64_t rows_per_mod, int64_t mod_ld, int group, int8_t* q, float* s,
                    void* stream) {
  if (M < 0 || K <= 0) return fail("ln_mod_quant: bad shape");
  if (M == 0) return DC_OK;
  if (x == nullptr || shift == nullptr || scale == nullptr || q == nullptr || s == nullptr)
    return fail("ln_mod_quant: null pointer");
  if (reinterpret_cast<uintptr_t>(s) % 4) return fail("ln_mod_quant: s must be 4-byte aligned");
  if (group != 0 && group != 256) return fail("ConvRot group must be 0 or 256 (got %d)", group);
  if (group && K % 256) return fail("K=%lld is not a multiple of the ConvRot group 256", (long long)K);
  if (K % 8 || K > 4096) return fail("ln_mod_quant: K must be a multiple of 8 and at most 4096");
  if (ldx < K || ldx % 8 || mod_ld % 8 || rows_per_mod <= 0) return fail("ln_mod_quant: bad strides");
  if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(shift) % 16 ||
      reinterpret_cast<uintptr_t>(scale) % 16 || reinterpret_cast<uintptr_t>(q) % 8)
    return fail("ln_mod_quant: x, shift, scale must be 16-byte and q 8-byte aligned");
  if (int r = check_sm100()) return r;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (K % 256 == 0 && rows_per_mod >= M && reinterpret_cast<uintptr_t>(q) % 16 == 0 &&
      (x_dtype == DC_DTYPE_BF16 || x_dtype == DC_DTYPE_F16)) {
    dc::RowSrc src = dc::plain_rows(x, ldx);
    src.full_div = quant_full_div();
    src.rot_order = dc::rot_order_for_width(K);
    if (x_dtype == DC_DTYPE_BF16)
      return group ? launch_rowq_warp<__nv_bfloat16, true, true, false>(src, M, K, shift, scale, q, s, st)
                   : launch_rowq_warp<__nv_bfloat16, false, true, false>(src, M, K, shift, scale, q, s, st);
    return group ? launch_rowq_warp<__half, true, true, false>(src, M, K, shift, scale, q, s, st)
                 : launch_rowq_warp<__half, false, true, false>(src, M, K, shift, scale, q, s, st);
  }
  switch (x_dtype) {
    case DC_DTYPE_BF16:
      return group ? launch_ln_mod_quant<__nv_bfloat16, true>(x, M, K, ldx, shift, scale, rows_per_mod, mod_ld, q, s, st)
                   : launch_ln_mod_quant<__nv_bfloat16, false>(x, M, K, ldx, shift, scale, rows_per_mod, mod_ld, q, s, st);
    case DC_DTYPE_F16:
      return group ? launch_ln_mod_quant<__half, true>(x, M, K, ldx, shift, scale, rows_per_mod, mod_ld, q, s, st)
                   : launch_ln_mod_quant<__half, false>(x, M, K, ldx, shift, scale, rows_per_mod, mod_ld, q, s, st);
    default: return fail("ln_mod_quant: dtype must be fp16 or bf16");
  }
}

static int qk_norm_rope_impl(void* qkv, int dtype, int64_t L, int64_t H, int64_t D, int64_t ld_row, int64_t q_off,
                             int64_t k_off, const void* q_scale0, const void* k_scale0, const void* q_scale1,
                             const void* k_scale1, int64_t split_row, const float* pe, int64_t pe_row0,
                             int8_t* q_codes, float* q_rscale, int64_t q_lpad, int write_q, void* stream) {
  if (L < 0 || H <= 0) return fail("qk_norm_rope: bad shape");
  if (q_codes != nullptr) {
    if (q_rscale == nullptr) return fail("qk_norm_rope: Q codes need their scale array");
    if (q_lpad < L) return fail("qk_norm_rope: q_lpad=%lld below L=%lld", (long long)q_lpad, (long long)L);
    if (reinterpret_cast<uintptr_t>(q_codes) % 4 || reinterpret_cast<uintptr_t>(q_rscale) % 4)
      return fail("qk_norm_rope: Q codes and scales must be 4-byte aligned");
  } else if (!write_q) {
    return fail("qk_norm_rope: write_q = 0 needs the Q codes output");
  }
  if (L == 0) return DC_OK;
  if (qkv == nullptr) return fail("qk_norm_rope: null qkv");
  if (D != 128) return fail("qk_norm_rope: head dim must be 128 (got %lld)", (long long)D);
  if (ld_row % 4 || q_off % 4 || k_off % 4 || reinterpret_cast<uintptr_t>(qkv) % 8)
    return fail("qk_norm_rope: rows and offsets must be 8-byte aligned");
  if (q_scale0 == nullptr || k_scale0 == nullptr || pe == nullptr) return fail("qk_norm_rope: scales and pe are required");
  if (split_row < L && (q_scale1 == nullptr || k_scale1 == nullptr)) return fail("qk_norm_rope: second scales missing");
  // scales are read 4 elements (8 bytes) per lane, pe 8 floats (two 16-byte loads) per lane
  for (const void* sp : {q_scale0, k_scale0, q_scale1, k_scale1})
    if (reinterpret_cast<uintptr_t>(sp) % 8) return fail("qk_norm_rope: scale vectors must be 8-byte aligned");
  if (reinterpret_cast<uintptr_t>(pe) % 16) return fail("qk_norm_rope: pe must be 16-byte aligned");
  if (pe_row0 < 0) return fail("qk_norm_rope: pe_row0 < 0");
  if (int r = check_sm100()) return r;
  dc::QkNormRopeParams p;
  p.qkv = qkv; p.L = L; p.H = H; p.ld_row = ld_row; p.q_off = q_off; p.k_off = k_off;
  p.q_scale[0] = q_scale0; p.k_scale[0] = k_scale0;
  p.q_scale[1] = q_scale1 ? q_scale1 : q_scale0; p.k_scale[1] = k_scale1 ? k_scale1 : k_scale0;
  p.split_row = split_row; p.pe = pe; p.pe_row0 = pe_row0;
  p.q_codes = q_codes; p.q_rscale = q_rscale; p.q_lpad = q_lpad; p.write_q = write_q;
  if (L * 2 * H >= (int64_t(1) << 31)) return fail("qk_norm_rope: L * 2H must stay below 2^31");
  // one warp per (row, vector); the Q-code padding rows need CTAs too
  const int64_t warps = L * 2 * H;
  int64_t want = (warps + dc::kRopeWarps - 1) / dc::kRopeWarps;
  if (q_codes != nullptr && q_lpad - L > want) want = q_lpad - L;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  const int ctas = static_cast<int>(want < cap ? want : cap);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  constexpr int threads = 32 * dc::kRopeWarps;
  if (dtype == DC_DTYPE_BF16) dc::qk_norm_rope_kernel<__nv_bfloat16><<<ctas, threads, 0, st>>>(p);
  else if (dtype == DC_DTYPE_F16) dc::qk_norm_rope_kernel<__half><<<ctas, threads, 0, st>>>(p);
  else return fail("qk_norm_rope: dtype must be fp16 or bf16");
  DC_CHECK_LAUNCH("qk_norm_rope launch");
  return DC_OK;
}

int dc_qk_norm_rope(void* qkv, int dtype, int64_t L, int64_t H, int64_t D, int64_t ld_row, int64_t q_off,
                    int64_t k_off, const void* q_scale0, const void* k_scale0, const void* q_scale1,
                    const void* k_scale1, int64_t split_row, const float* pe, int64_t pe_row0, void* stream) {
  return qk_norm_rope_impl(qkv, dtype, L, H, D, ld_row, q_off, k_off, q_scale0, k_scale0, q_scale1, k_scale1,
                           split_row, pe, pe_row0, nullptr, nullptr, 0, 1, stream);
}

int dc_qk_norm_rope_q8(void* qkv, int dtype, int64_t L, int64_t H, int64_t D, int64_t ld_row, int64_t q_off,
                       int64_t k_off, const void* q_scale0, const void* k_scale0, const void* q_scale1,
                       const void* k_scale1, int64_t split_row, const float* pe, int64_t pe_row0, int8_t* q_codes,
                       float* q_rscale, int64_t q_lpad, int write_q, void* stream) {
  if (q_codes == nullptr) return fail("qk_norm_rope_q8: null Q codes");
  return qk_norm_rope_impl(qkv, dtype, L, H, D, ld_row, q_off, k_off, q_scale0, k_scale0, q_scale1, k_scale1,
                           split_row, pe, pe_row0, q_codes, q_rscale, q_lpad, write_q, stream);
}

int dc_rescale(const int32_t* acc, int64_t lda, const float* sx, const float* sw, const void* bias, void* out,
               int64_t ldo, int out_dtype, int64_t M, int64_t N, void* stream) {
  if (M < 0 || N <= 0) return fail("rescale: bad shape");
  if (M == 0) return DC_OK;
  if (lda < N || ldo < N) return fail("rescale: leading dimension smaller than the row");
  if (M > INT32_MAX || N > INT32_MAX) return fail("rescale: dimension above 2^31");
  if (acc == nullptr || sx == nullptr || sw == nullptr || out == nullptr) return fail("rescale: null pointer");
  if (reinterpret_cast<uintptr_t>(acc) % 4 || reinterpret_cast<uintptr_t>(sx) % 4 ||
      reinterpret_cast<uintptr_t>(sw) % 4 || reinterpret_cast<uintptr_t>(out) % 2 ||
      reinterpret_cast<uintptr_t>(bias) % 2)
    return fail("rescale: pointers must be aligned to their element size");
  if (int r = check_sm100()) return r;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int grid = static_cast<int>(M < 4096 ? M : 4096);
  if (out_dtype == DC_DTYPE_BF16)
    dc::rescale_kernel<dc::kOutBF16><<<grid, 256, 0, st>>>(acc, lda, sx, sw, bias, out, ldo, static_cast<int>(M), static_cast<int>(N));
  else if (out_dtype == DC_DTYPE_F16)
    dc::rescale_kernel<dc::kOutF16><<<grid, 256, 0, st>>>(acc, lda, sx, sw, bias, out, ldo, static_cast<int>(M), static_cast<int>(N));
  else
    return fail("rescale: output dtype must be fp16 or bf16");
  DC_CHECK_LAUNCH("rescale launch");
  return DC_OK;
}

int dc_attn_workspace_size(int64_t B, int64_t H, int64_t Lq, int64_t Lk, int64_t D, int mode, size_t* bytes) {
  if (int r = check_attn_args(DC_DTYPE_BF16, B, H, Lq, Lk, D, mode)) return r;
  *bytes = attn_layout(B, H, Lq, Lk, D, mode).total;
  return DC_OK;
}

int dc_attn_workspace_layout(int64_t B, int64_t H, int64_t Lq, int64_t Lk, int64_t D, int mode, int64_t* out8) {
  if (int r = check_attn_args(DC_DTYPE_BF16, B, H, Lq, Lk, D, mode)) return r;
  AttnLayout a = attn_layout(B, H, Lq, Lk, D, mode);
  out8[0] = a.Lq_pad; out8[1] = a.Lk_pad;
  out8[2] = static_cast<int64_t>(a.q_codes); out8[3] = static_cast<int64_t>(a.k_codes);
  out8[4] = static_cast<int64_t>(a.q_scale); out8[5] = static_cast<int64_t>(a.k_scale);
  out8[6] = static_cast<int64_t>(a.ksum); out8[7] = static_cast<int64_t>(a.total);
  return DC_OK;
}

static int attn_common(bool run_prep, bool run_main, const void* q, const void* k, const void* v, int dtype, int64_t B, int64_t H,
                       int64_t Lq, int64_t Lk, int64_t D, const int64_t* q_strides, const int64_t* k_strides,
                       const int64_t* v_strides, float sm_scale, int mode, void* o, const int64_t* o_strides,
                       void* workspace, size_t ws_bytes, void* stream, bool prep_q = true) {
  if (int r = check_attn_args(dtype, B, H, Lq, Lk, D, mode)) return r;
  if (run_prep) {
    if (prep_q)
      if (int r = check_strides(q, q_strides, "q")) return r;
    if (int r = check_strides(k, k_strides, "k")) return r;
  }
  if (run_main) {
    if (int r = check_strides(v, v_strides, "v")) return r;
    if (int r = check_strides(o, o_strides, "o")) return r;
  }
  AttnLayout a = attn_layout(B, H, Lq, Lk, D, mode);
  if (workspace == nullptr || ws_bytes < a.total)
    return fail("attention workspace too small: need %zu bytes, got %zu", a.total, ws_bytes);
  if (reinterpret_cast<uintptr_t>(workspace) % 256 != 0) return fail("attention workspace must be 256-byte aligned");
  if (int r = check_sm100()) return r;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int r = DC_OK;
  if (dtype == DC_DTYPE_BF16) {
    if (run_prep)
      r = D == 128 ? attn_prep<__nv_bfloat16, 128>(q, k, B, H, Lq, Lk, q_strides, k_strides, mode, ws, a, st, prep_q)
                   : attn_prep<__nv_bfloat16, 64>(q, k, B, H, Lq, Lk, q_strides, k_strides, mode, ws, a, st, prep_q);
    if (r || !run_main) return r;
    return D == 128 ? attn_main<__nv_bfloat16, 128>(v, B, H, Lq, Lk, v_strides, sm_scale, o, o_strides, ws, a, st)
                    : attn_main<__nv_bfloat16, 64>(v, B, H, Lq, Lk, v_strides, sm_scale, o, o_strides, ws, a, st);
  }
  if (run_prep)
    r = D == 128 ? attn_prep<__half, 128>(q, k, B, H, Lq, Lk, q_strides, k_strides, mode, ws, a, st, prep_q)
                 : attn_prep<__half, 64>(q, k, B, H, Lq, Lk, q_strides, k_strides, mode, ws, a, st, prep_q);
  if (r || !run_main) return r;
  return D == 128 ? attn_main<__half, 128>(v, B, H, Lq, Lk, v_strides, sm_scale, o, o_strides, ws, a, st)
                  : attn_main<__half, 64>(v, B, H, Lq, Lk, v_strides, sm_scale, o, o_strides, ws, a, st);
}

int dc_attn_int8_fwd(const void* q, const void* k, const void* v, int dtype, int64_t B, int64_t H, int64_t Lq,
                     int64_t Lk, int64_t D, const int64_t* q_strides, const int64_t* k_strides,
                     const int64_t* v_strides, float sm_scale, int mode, void* o, const int64_t* o_strides,
                     void* workspace, size_t workspace_bytes, void* stream) {
  return attn_common(true, true, q, k, v, dtype, B, H, Lq, Lk, D, q_strides, k_strides, v_strides, sm_scale, mode,
                     o, o_strides, workspace, workspace_bytes, stream);
}

int dc_attn_int8_main(const void* v, int dtype, int64_t B, int64_t H, int64_t Lq, int64_t Lk, int64_t D,
                      const int64_t* v_strides, float sm_scale, int mode, void* o, const int64_t* o_strides,
                      void* workspace, size_t workspace_bytes, void* stream) {
  return attn_common(false, true, nullptr, nullptr, v, dtype, B, H, Lq, Lk, D, nullptr, nullptr, v_strides, sm_scale,
                     mode, o, o_strides, workspace, workspace_bytes, stream);
}

int dc_attn_int8_prep(const void* q, const void* k, int dtype, int64_t B, int64_t H, int64_t Lq, int64_t Lk,
                      int64_t D, const int64_t* q_strides, const int64_t* k_strides, int mode, void* workspace,
                      size_t workspace_bytes, void* stream) {
  return attn_common(true, false, q, k, nullptr, dtype, B, H, Lq, Lk, D, q_strides, k_strides, nullptr, 1.0f, mode,
                     nullptr, nullptr, workspace, workspace_bytes, stream);
}

int dc_attn_int8_prep_k(const void* k, int dtype, int64_t B, int64_t H, int64_t Lq, int64_t Lk, int64_t D,
                        const int64_t* k_strides, int mode, void* workspace, size_t workspace_bytes, void* stream) {
  return attn_common(true, false, nullptr, k, nullptr, dtype, B, H, Lq, Lk, D, nullptr, k_strides, nullptr, 1.0f, mode,
                     nullptr, nullptr, workspace, workspace_bytes, stream, false);
}

int dc_attn_split_partials_size(int64_t B, int64_t H, int64_t Lq, int64_t Lk, int64_t D, int nsplit, size_t* bytes) {
  if (bytes == nullptr) return fail("attn_split_partials_size: null output");
  if (int r = check_attn_args(DC_DTYPE_BF16, B, H, Lq, Lk, D, dc::kModeRef)) return r;
  const AttnLayout a = attn_layout(B, H, Lq, Lk, D, dc::kModeRef);
  const int64_t n = a.Lk_pad / dc::kAttnBN;
  if (nsplit < 1 || nsplit > n) return fail("nsplit=%d must be in [1, %lld] (key tiles of 128)", nsplit, (long long)n);
  int tps = 0, ranges = 0;
  split_ranges(n, nsplit, &tps, &ranges);
  *bytes = split_partial_bytes(B * H, a.Lq_pad, D, ranges);
  return DC_OK;
}

int dc_attn_int8_main_split(const void* v, int dtype, int64_t B, int64_t H, int64_t Lq, int64_t Lk, int64_t D,
                            const int64_t* v_strides, float sm_scale, int mode, void* o, const int64_t* o_strides,
                            void* workspace, size_t workspace_bytes, int nsplit, void* partials,
                            size_t partial_bytes, void* stream) {
  if (int r = check_attn_args(dtype, B, H, Lq, Lk, D, mode)) return r;
  if (int r = check_strides(v, v_strides, "v")) return r;
  if (int r = check_strides(o, o_strides, "o")) return r;
  const AttnLayout a = attn_layout(B, H, Lq, Lk, D, mode);
  if (workspace == nullptr || workspace_bytes < a.total)
    return fail("attention workspace too small: need %zu bytes, got %zu", a.total, workspace_bytes);
  if (reinterpret_cast<uintptr_t>(workspace) % 256 != 0) return fail("attention workspace must be 256-byte aligned");
  const int64_t n = a.Lk_pad / dc::kAttnBN;
  if (nsplit < 1 || nsplit > n) return fail("nsplit=%d must be in [1, %lld] (key tiles of 128)", nsplit, (long long)n);
  if (B * H > INT32_MAX / 2) return fail("split attention: B*H too large");
  int tps = 0, ranges = 0;
  split_ranges(n, nsplit, &tps, &ranges);
  const size_t need = split_partial_bytes(B * H, a.Lq_pad, D, ranges);
  if (partials == nullptr || partial_bytes < need)
    return fail("split attention partials too small: need %zu bytes, got %zu", need, partial_bytes);
  if (reinterpret_cast<uintptr_t>(partials) % 256 != 0) return fail("split attention partials must be 256-byte aligned");
  if (int r = check_sm100()) return r;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (dtype == DC_DTYPE_BF16)
    return D == 128 ? attn_main_split<__nv_bfloat16, 128>(v, B, H, Lq, Lk, v_strides, sm_scale, o, o_strides, ws, a,
                                                          nsplit, partials, st)
                    : attn_main_split<__nv_bfloat16, 64>(v, B, H, Lq, Lk, v_strides, sm_scale, o, o_strides, ws, a,
                                                         nsplit, partials, st);
  return D == 128 ? attn_main_split<__half, 128>(v, B, H, Lq, Lk, v_strides, sm_scale, o, o_strides, ws, a, nsplit,
                                                 partials, st)
                  : attn_main_split<__half, 64>(v, B, H, Lq, Lk, v_strides, sm_scale, o, o_strides, ws, a, nsplit,
                                                partials, st);
}

// ---------------------------------------------------------------------------------------------
// Attention for callers that cannot allocate device memory: an application that owns every byte
// of GPU memory through its own pool and has no way to hand this library a workspace, or that
// calls at a point where cudaMalloc's implicit device synchronization is not allowed. The Q/K
// codes and scales the attention needs between its two stages live instead in one fixed
// file-scope device array. Every GPU that loads this library holds that array (kNoAllocScratch
// bytes) until the process exits.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratch];

namespace {
std::mutex g_noalloc_mutex;
void* g_noalloc_addr[256] = {};   // device address of g_noalloc_scratch, per device ordinal
void* g_noalloc_ctx[256] = {};    // the CUDA context that address belongs to

// The current CUDA context (cuCtxGetCurrent through the runtime's driver entry point), or null.
void* current_context() {
  typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  CUcontext ctx = nullptr;
  if (fn == nullptr || fn(&ctx) != CUDA_SUCCESS) return nullptr;
  return ctx;
}

// The scratch array's device address for the current device. In host code the array's name is
// only a host-side stand-in, so the address comes from cudaGetSymbolAddress with that device
// current: on the first call on each device, and again whenever the device's context is not the
// one the address was looked up in (after cudaDeviceReset the module is loaded anew and the array
// may sit elsewhere).
int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 256) return fail("device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  void* ctx = current_context();
  if (g_noalloc_addr[dev] == nullptr || ctx == nullptr || ctx != g_noalloc_ctx[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(scratch)");
    g_noalloc_addr[dev] = p;
    g_noalloc_ctx[dev] = current_context();   // the lookup made the primary context current if none was
  }
  *out = g_noalloc_addr[dev];
  return DC_OK;
}
}  // namespace

int dc_attn_int8_fwd_noalloc(const void* q, const void* k, const void* v, int dtype, int64_t B, int64_t H,
                             int64_t Lq, int64_t Lk, int64_t D, const int64_t* q_strides, const int64_t* k_strides,
                             const int64_t* v_strides, float sm_scale, int mode, void* o, const int64_t* o_strides,
                             void* stream) {
  if (int r = check_attn_args(dtype, B, H, Lq, Lk, D, mode)) return r;
  const size_t need = attn_layout(B, H, Lq, Lk, D, mode).total;
  if (need > kNoAllocScratch)
    return fail("attention without allocation: these shapes need %zu bytes of scratch, the fixed scratch "
                "holds %zu (B*H*(Lq + Lk)*D ~ 32 MiB at most); use dc_attn_int8_fwd with a workspace",
                need, kNoAllocScratch);
  if (int r = check_sm100()) return r;
  void* scratch = nullptr;
  if (int r = noalloc_scratch(&scratch)) return r;
  // Nothing in the scratch has to start at zero: each call writes every byte it later reads.
  return attn_common(true, true, q, k, v, dtype, B, H, Lq, Lk, D, q_strides, k_strides, v_strides, sm_scale, mode,
                     o, o_strides, scratch, kNoAllocScratch, stream);
}

int dc_selftest_exp2(const float* x, float* poly, float* ref, int64_t n, void* stream) {
  if (n < 2 || n % 2 || n > (1 << 30)) return fail("selftest_exp2: n must be even, 2 <= n <= 2^30");
  if (int r = check_sm100()) return r;
  const int threads = 256;
  const int blocks = static_cast<int>((n / 2 + threads - 1) / threads);
  selftest_exp2_kernel<<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(x, poly, ref, static_cast<int>(n));
  DC_CHECK_LAUNCH("selftest_exp2 launch");
  return DC_OK;
}

int dc_selftest_wait_timeout(long long limit_cycles, int* status_dev, void* stream) {
  if (limit_cycles <= 0 || limit_cycles > 4000000000LL) return fail("limit_cycles out of range");
  if (int r = check_sm100()) return r;
  selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(limit_cycles, status_dev);
  DC_CHECK_LAUNCH("selftest launch");
  return DC_OK;
}

}  // extern "C"
