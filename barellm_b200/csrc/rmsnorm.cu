// Residual add + RMSNorm of the decoder that drives the paged-attention path
// (decoder support; not one of the paged-KV kernels).  Replaces the chain of
// tensor ops of the reference's RMSNorm (src/barellm/models/norm.py:14-21)
//   xf = x.float(); xf * rsqrt(mean(xf^2) + eps); (xf * weight).to(x.dtype)
// and, with a residual, the add before it (models/block.py):
//   x_out = x + residual;  out = rmsnorm(x_out) * weight
// Roundings follow the tensor ops: the add rounded to the element type, the
// mean square, rsqrt and both products in fp32, one rounding at the end; only
// the mean square's summation order differs.
//
// One warp per row.  Pass 1 reads the row (and the residual), writes x_out
// and sums the squares; pass 2 reads the row again (now in L1/L2) and writes
// the normalised row.  16-byte vectors when every base and stride allows.
// Roofline: HBM / latency.  Bytes per row: hidden * E * (1 + [1 residual] +
// [1 x_out] + 1 out).
#include "common.cuh"

namespace bl {
namespace {

constexpr int kNormWarps = 8;

struct NormArgs {
  const void* x;
  const void* r;
  void* xo;
  void* out;
  const void* w;
  int64_t rows, hidden, xs, rs, xos, os;
  float eps;
};

template <typename T, bool VEC>
__device__ __forceinline__ void load8(const T* p, float (&v)[8], int n) {
  if constexpr (VEC) {
    constexpr int N = 16 / (int)sizeof(T);
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = to_f32<T>(e[i]);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i < n) v[i] = to_f32<T>(p[i]);
  }
}

template <typename T, bool VEC>
__device__ __forceinline__ void store8(T* p, const float (&v)[8], int n) {
  if constexpr (VEC) {
    constexpr int N = 16 / (int)sizeof(T);
    uint4 u;
    T* e = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int i = 0; i < N; ++i) e[i] = from_f32<T>(v[i]);
    *reinterpret_cast<uint4*>(p) = u;
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i < n) p[i] = from_f32<T>(v[i]);
  }
}

// grid: ceil(rows / 8) blocks of 8 warps; warp w of block x normalises row x * 8 + w
template <typename T, bool VEC, bool RES>
__global__ void __launch_bounds__(kNormWarps * 32) rms_norm_kernel(const NormArgs a) {
  constexpr int N = VEC ? 16 / (int)sizeof(T) : 8;  // elements per lane per step
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kNormWarps + (threadIdx.x >> 5);
  if (row >= a.rows) return;
  const T* x = reinterpret_cast<const T*>(a.x) + row * a.xs;
  const T* r = RES ? reinterpret_cast<const T*>(a.r) + row * a.rs : nullptr;
  T* xo = RES && a.xo ? reinterpret_cast<T*>(a.xo) + row * a.xos : nullptr;
  T* out = reinterpret_cast<T*>(a.out) + row * a.os;
  const T* w = reinterpret_cast<const T*>(a.w);
  const int64_t h = a.hidden;

  float ss = 0.f;
  for (int64_t c = (int64_t)lane * N; c < h; c += 32 * N) {
    const int n = h - c < N ? (int)(h - c) : N;
    float v[8];
    load8<T, VEC>(x + c, v, n);
    if (RES) {
      float u[8];
      load8<T, VEC>(r + c, u, n);
#pragma unroll
      for (int i = 0; i < N; ++i)
        if (i < n) v[i] = to_f32<T>(from_f32<T>(__fadd_rn(v[i], u[i])));
      if (xo) store8<T, VEC>(xo + c, v, n);
    }
#pragma unroll
    for (int i = 0; i < N; ++i)
      if (i < n) ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
  const float rs = rsqrtf(__fadd_rn(ss / (float)h, a.eps));

  for (int64_t c = (int64_t)lane * N; c < h; c += 32 * N) {
    const int n = h - c < N ? (int)(h - c) : N;
    float v[8], wv[8];
    load8<T, VEC>(x + c, v, n);
    if (RES) {
      float u[8];
      load8<T, VEC>(r + c, u, n);
#pragma unroll
      for (int i = 0; i < N; ++i)
        if (i < n) v[i] = to_f32<T>(from_f32<T>(__fadd_rn(v[i], u[i])));
    }
    load8<T, VEC>(w + c, wv, n);
#pragma unroll
    for (int i = 0; i < N; ++i)
      if (i < n) v[i] = __fmul_rn(__fmul_rn(v[i], rs), wv[i]);
    store8<T, VEC>(out + c, v, n);
  }
}

template <typename T>
int launch(const NormArgs& k, bool vec, bool res, cudaStream_t s) {
  const unsigned grid = (unsigned)((k.rows + kNormWarps - 1) / kNormWarps);
  const int threads = kNormWarps * 32;
  if (vec && res) rms_norm_kernel<T, true, true><<<grid, threads, 0, s>>>(k);
  else if (vec) rms_norm_kernel<T, true, false><<<grid, threads, 0, s>>>(k);
  else if (res) rms_norm_kernel<T, false, true><<<grid, threads, 0, s>>>(k);
  else rms_norm_kernel<T, false, false><<<grid, threads, 0, s>>>(k);
  BL_CHECK_LAUNCH("rms_norm_kernel");
  return BL_OK;
}

}  // namespace
}  // namespace bl

using namespace bl;

extern "C" int bl_rms_norm(const bl_rms_norm_args* args, void* stream) {
  BL_CHECK_ARG(args != nullptr, "bl_rms_norm: args is null");
  const bl_rms_norm_args& a = *args;
  BL_CHECK_ARG(a.x && a.out && a.weight, "bl_rms_norm: null pointer argument");
  BL_CHECK_ARG(a.rows > 0 && a.hidden > 0, "bl_rms_norm: rows and hidden must be positive");
  BL_CHECK_ARG(a.dtype == BL_F32 || a.dtype == BL_F16 || a.dtype == BL_BF16, "bl_rms_norm: unsupported dtype");
  BL_CHECK_ARG(!a.x_out || a.residual, "bl_rms_norm: x_out needs a residual");
  BL_CHECK_ARG((a.rows + kNormWarps - 1) / kNormWarps <= INT32_MAX, "bl_rms_norm: too many rows");
  const int64_t es = elem_size(a.dtype);
  NormArgs k;
  k.x = a.x;
  k.r = a.residual;
  k.xo = a.x_out;
  k.out = a.out;
  k.w = a.weight;
  k.rows = a.rows;
  k.hidden = a.hidden;
  k.xs = a.x_stride;
  k.rs = a.residual_stride;
  k.xos = a.x_out_stride;
  k.os = a.out_stride;
  k.eps = a.eps;
  // 16-byte vectors when the row length, every base and every row stride allow
  bool vec = (a.hidden * es) % 16 == 0;
  const void* bases[] = {a.x, a.residual, a.x_out, a.out, a.weight};
  for (const void* p : bases) vec = vec && (uint64_t)(uintptr_t)p % 16 == 0;
  for (int64_t st : std::initializer_list<int64_t>{a.x_stride, a.residual_stride, a.x_out_stride, a.out_stride})
    vec = vec && (uint64_t)(st * es) % 16 == 0;
  const bool res = a.residual != nullptr;
  cudaStream_t s = (cudaStream_t)stream;
  switch (a.dtype) {
    case BL_F32: return launch<float>(k, vec, res, s);
    case BL_F16: return launch<__half>(k, vec, res, s);
    default: return launch<__nv_bfloat16>(k, vec, res, s);
  }
}
