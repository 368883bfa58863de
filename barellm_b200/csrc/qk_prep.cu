// Fused QK-RMSNorm + RoPE + paged append: the step just before the paged
// attention, in one launch.
//
// Replaces, per layer, the reference chain (src/barellm/models/attention.py:
// 161-169 with models/norm.py:14-21 and models/rope.py:53-68)
//   q = apply_rope(q_norm(q), cos, sin); k = apply_rope(k_norm(k), cos, sin)
// followed by PagedLayerKV.append_only of k and v
// (src/barellm/engine/paged_kv_cache.py:151-193):
//   q_out[b, hq, t]           = rope(rmsnorm(q_in[b, hq, t]) * q_w)
//   K slot (b, start_b + t, h) = rope(rmsnorm(k_in[b, h, t]) * k_w)
//   V slot (b, start_b + t, h) = v_in[b, h, t]
// Rounding follows the reference's tensor ops: the mean square, rsqrt and the
// weight product in fp32 with one rounding to the element type; RoPE's
// x * cos and rotate_half(x) * sin each rounded to the element type and their
// sum rounded again (no fused multiply-add, as separate tensor ops have none).
// The only difference is the summation order of the mean square.
//
// Work layout: a half-warp owns one row kind (one q, k or v head) of a block
// of 16 consecutive tokens of one request, and lane l of the half holds
// elements [E*l, E*l + E) of the row (E = D / 16, one 16-byte vector at
// D = 128 in bf16), so RoPE's partner element d +- D/2 sits in lane l ^ 8 and
// the norm's sum is a 4-step shuffle inside the half.  The 16-bit types do
// their arithmetic on fp32 pairs (mul / add .f32x2) with the roundings on
// packed pairs.  With VEC every lane moves its E elements as one vector (the
// caller checks the alignment of every base and stride).
// Roofline: HBM.  Bytes per token: (Hq + 2 Hkv) * D * E_in read,
// (Hq + 2 Hkv) * D * E written, plus one cos and one sin row.
#include <type_traits>

#include "common.cuh"

namespace bl {
namespace {

constexpr int kWarps = 8;
constexpr int kTokTile = 16;  // tokens per block
constexpr int kTok = 4;       // tokens per half-warp pass, their row loads in flight together

struct PrepArgs {
  const void* q_in;
  int64_t qi_sb, qi_sh, qi_st;
  const void* k_in;
  int64_t ki_sb, ki_sh, ki_st;
  const void* v_in;
  int64_t vi_sb, vi_sh, vi_st;
  void* q_out;
  int64_t qo_sb, qo_sh, qo_st;
  const void* qw;
  const void* kw;
  const void* cos;
  const void* sin;
  int64_t rope_sb, rope_st;
  float eps;
  int32_t hq, hkv;
  void* k_pool;
  void* v_pool;
  int64_t num_blocks, layer;
  int32_t bs, bs_shift;  // bs_shift >= 0 when bs is a power of two
  const int32_t* block_tables;
  int64_t bt_stride;
  int32_t bt_width;
  const int32_t* row_ids;
  const int32_t* start_pos;
  const int32_t* new_offsets;
  int32_t max_new;
  int32_t* err;
};

template <int BYTES> struct VecOf;
template <> struct VecOf<4> { using type = uint32_t; };
template <> struct VecOf<8> { using type = uint2; };
template <> struct VecOf<16> { using type = uint4; };
template <> struct VecOf<32> { struct alignas(16) type { uint4 a, b; }; };
template <> struct VecOf<64> { struct alignas(16) type { uint4 a, b, c, d; }; };

// E consecutive elements at p into fp32 registers (one vector load with VEC)
template <typename T, int E, bool VEC>
__device__ __forceinline__ void load_e(const T* p, float (&x)[E]) {
  if constexpr (VEC) {
    using V = typename VecOf<E * (int)sizeof(T)>::type;
    const V v = *reinterpret_cast<const V*>(p);
    const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
    for (int i = 0; i < E; ++i) x[i] = to_f32<T>(e[i]);
  } else {
#pragma unroll
    for (int i = 0; i < E; ++i) x[i] = to_f32<T>(p[i]);
  }
}

template <typename T, int E, bool VEC>
__device__ __forceinline__ void store_e(T* p, const float (&x)[E]) {
  if constexpr (VEC) {
    using V = typename VecOf<E * (int)sizeof(T)>::type;
    V v;
    T* e = reinterpret_cast<T*>(&v);
#pragma unroll
    for (int i = 0; i < E; ++i) e[i] = from_f32<T>(x[i]);
    *reinterpret_cast<V*>(p) = v;
  } else {
#pragma unroll
    for (int i = 0; i < E; ++i) p[i] = from_f32<T>(x[i]);
  }
}

template <typename T>
__device__ __forceinline__ float round_to(float x) {
  return to_f32<T>(from_f32<T>(x));
}

// the pair (x[i], x[i+1]) rounded to T, back in fp32
template <typename T>
__device__ __forceinline__ float2 round2(uint64_t v) {
  const float2 f = f2_unpack(v);
  return unpack2<T>(pack2<T>(f.x, f.y));
}

// rope(rmsnorm(x) * w) in place, the reference's roundings (see the file header)
// rope(rmsnorm(x) * w) of one row held by a half-warp (E elements per lane,
// lane `sub` of the half holds elements [E*sub, E*sub + E)); w, cos and sin
// are read from shared memory.  The reference's roundings (file header).
// rope(rmsnorm(x) * w) of one row held by a half-warp (E elements per lane,
// lane `sub` of the half holds elements [E*sub, E*sub + E)), the reference's
// roundings (file header).  w, cos and sin are this lane's E elements.
template <typename T, int E>
__device__ __forceinline__ void norm_rope(float (&x)[E], const float (&w)[E], const float (&cs)[E],
                                          const float (&sn)[E], float eps, int sub, unsigned hmask) {
  constexpr int D = 16 * E;
  if constexpr (std::is_same_v<T, float>) {
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) ss = __fadd_rn(ss, __fmul_rn(x[e], x[e]));
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(hmask, ss, o));
    const float rs = rsqrtf(__fadd_rn(ss / (float)D, eps));
#pragma unroll
    for (int e = 0; e < E; ++e) x[e] = __fmul_rn(__fmul_rn(x[e], rs), w[e]);
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float partner = __shfl_xor_sync(hmask, x[e], 8);
      const float rot = sub < 8 ? -partner : partner;
      x[e] = __fadd_rn(__fmul_rn(x[e], cs[e]), __fmul_rn(rot, sn[e]));
    }
  } else {
    constexpr int P = E / 2;
    uint64_t acc = f2_pack(0.f, 0.f);
#pragma unroll
    for (int p = 0; p < P; ++p) {
      const uint64_t v = f2_pack(x[2 * p], x[2 * p + 1]);
      acc = f2_add(acc, f2_mul(v, v));
    }
    const float2 a2 = f2_unpack(acc);
    float ss = __fadd_rn(a2.x, a2.y);
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(hmask, ss, o));
    const float rs = rsqrtf(__fadd_rn(ss / (float)D, eps));
    const uint64_t rs2 = f2_pack(rs, rs);
    const uint32_t neg = sub < 8 ? 0x80008000u : 0u;  // rotate_half negates the upper half's partner
#pragma unroll
    for (int p = 0; p < P; ++p) {
      // norm: one rounding after the weight
      const float2 y = f2_unpack(f2_mul(f2_mul(f2_pack(x[2 * p], x[2 * p + 1]), rs2), f2_pack(w[2 * p], w[2 * p + 1])));
      const uint32_t yp = pack2<T>(y.x, y.y);
      // partner pair (elements d +- D/2) from lane ^ 8, negated for the lower lanes
      const uint32_t rp = __shfl_xor_sync(hmask, yp, 8) ^ neg;
      const float2 yf = unpack2<T>(yp), rf = unpack2<T>(rp);
      const float2 xc = round2<T>(f2_mul(f2_pack(yf.x, yf.y), f2_pack(cs[2 * p], cs[2 * p + 1])));
      const float2 rsn = round2<T>(f2_mul(f2_pack(rf.x, rf.y), f2_pack(sn[2 * p], sn[2 * p + 1])));
      const float2 o = f2_unpack(f2_add(f2_pack(xc.x, xc.y), f2_pack(rsn.x, rsn.y)));
      x[2 * p] = o.x;  // rounded to T by the store
      x[2 * p + 1] = o.y;
    }
  }
}

// A row slice as loaded: E elements' raw bits, converted to fp32 where used.
template <typename T, int E>
using RawE = typename VecOf<E * (int)sizeof(T)>::type;

template <typename T, int E, bool VEC>
__device__ __forceinline__ RawE<T, E> load_raw(const T* p) {
  RawE<T, E> r;
  if constexpr (VEC) {
    r = *reinterpret_cast<const RawE<T, E>*>(p);
  } else {
    T* e = reinterpret_cast<T*>(&r);
#pragma unroll
    for (int i = 0; i < E; ++i) e[i] = p[i];
  }
  return r;
}

template <typename T, int E>
__device__ __forceinline__ void raw_to_f32(const RawE<T, E>& r, float (&x)[E]) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(&r);
  if constexpr (std::is_same_v<T, float>) {
#pragma unroll
    for (int i = 0; i < E; ++i) x[i] = __uint_as_float(w[i]);
  } else {
#pragma unroll
    for (int i = 0; i < E / 2; ++i) {
      const float2 f = unpack2<T>(w[i]);
      x[2 * i] = f.x;
      x[2 * i + 1] = f.y;
    }
  }
}

// bf16 pair arithmetic, one rounding per operation (PTX mul / add .rn.bf16x2).
// For bf16 inputs these equal the fp32 operation followed by a rounding to
// bf16: a product of two bf16 values is exact in fp32, and a sum that fp32
// has to round differs from the exact one by far less than half a bf16 step.
__device__ __forceinline__ uint32_t bf2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t bf2_add(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// norm_rope for bf16 rows kept as packed pairs: the norm in fp32 pairs, RoPE's
// round(round(y * cos) + round(rot * sin)) on bf16 pairs.  x / cs / sn: E / 2
// words of this lane's elements; x is replaced by the result.
template <int E>
__device__ __forceinline__ void norm_rope_bf16(uint32_t (&x)[E / 2], const float (&w)[E], const uint32_t (&cs)[E / 2],
                                               const uint32_t (&sn)[E / 2], float eps, int sub, unsigned hmask) {
  constexpr int D = 16 * E;
  constexpr int P = E / 2;
  float xf[E];
#pragma unroll
  for (int p = 0; p < P; ++p) {
    const float2 f = unpack2<__nv_bfloat16>(x[p]);
    xf[2 * p] = f.x;
    xf[2 * p + 1] = f.y;
  }
  uint64_t acc = f2_pack(0.f, 0.f);
#pragma unroll
  for (int p = 0; p < P; ++p) {
    const uint64_t v = f2_pack(xf[2 * p], xf[2 * p + 1]);
    acc = f2_add(acc, f2_mul(v, v));
  }
  const float2 a2 = f2_unpack(acc);
  float ss = __fadd_rn(a2.x, a2.y);
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(hmask, ss, o));
  const float rs = rsqrtf(__fadd_rn(ss / (float)D, eps));
  const uint64_t rs2 = f2_pack(rs, rs);
  const uint32_t neg = sub < 8 ? 0x80008000u : 0u;  // rotate_half negates the upper half's partner
#pragma unroll
  for (int p = 0; p < P; ++p) {
    const float2 y = f2_unpack(f2_mul(f2_mul(f2_pack(xf[2 * p], xf[2 * p + 1]), rs2), f2_pack(w[2 * p], w[2 * p + 1])));
    const uint32_t yp = pack2<__nv_bfloat16>(y.x, y.y);  // norm: one rounding after the weight
    const uint32_t rp = __shfl_xor_sync(hmask, yp, 8) ^ neg;
    x[p] = bf2_add(bf2_mul(yp, cs[p]), bf2_mul(rp, sn[p]));
  }
}

template <typename T, int E>
__device__ __forceinline__ void raw_words(const RawE<T, E>& r, uint32_t (&w)[E * (int)sizeof(T) / 4]) {
  const uint32_t* p = reinterpret_cast<const uint32_t*>(&r);
#pragma unroll
  for (int i = 0; i < E * (int)sizeof(T) / 4; ++i) w[i] = p[i];
}

template <typename T, int E, bool VEC>
__device__ __forceinline__ void store_words(T* p, const uint32_t (&w)[E * (int)sizeof(T) / 4]) {
  RawE<T, E> r;
  uint32_t* q = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
  for (int i = 0; i < E * (int)sizeof(T) / 4; ++i) q[i] = w[i];
  if constexpr (VEC) {
    *reinterpret_cast<RawE<T, E>*>(p) = r;
  } else {
    const T* e = reinterpret_cast<const T*>(&r);
#pragma unroll
    for (int i = 0; i < E; ++i) p[i] = e[i];
  }
}

// Grid (ceil(max_new / kTokTile), batch, ceil(row pairs / 8)).  Half-warp
// `half` of warp w owns one row kind for the whole block -- row
// j = 2 * (blockIdx.z * 8 + w) + half, a q, k or v head -- and walks the block's
// kTokTile tokens, kTok at a time with their row loads in flight together.
// Its norm weights stay in registers; the block's cos / sin rows are staged
// in shared memory once (the first rows' loads are issued before that
// barrier); k / v rows look up their token's pool slot.
template <typename T, int E, bool VEC>
__global__ void __launch_bounds__(kWarps * 32, E <= 8 ? 4 : 2) qk_prep_kernel(const PrepArgs a) {
  constexpr int D = 16 * E;
  __shared__ __align__(16) T s_rope[2][kTokTile][D];  // cos, sin of the block's tokens
  const int lane = threadIdx.x & 31;
  const int half = lane >> 4, sub = lane & 15;
  const unsigned hmask = half ? 0xffff0000u : 0x0000ffffu;
  const int j = 2 * (blockIdx.z * kWarps + (threadIdx.x >> 5)) + half;
  const int heads = a.hq + 2 * a.hkv;
  const bool active = j < heads;  // half-warp uniform; inactive halves still meet the barrier
  const int b = blockIdx.y;
  int n_b = a.max_new, o_b = 0;
  if (a.new_offsets) {
    o_b = a.new_offsets[b];
    n_b = a.new_offsets[b + 1] - o_b;
  }
  const int t0 = blockIdx.x * kTokTile;
  const int t_end = min(t0 + kTokTile, n_b);
  if (t0 >= t_end) return;  // block-uniform
  const int64_t bi = a.new_offsets ? 0 : b;  // packed inputs have one batch row
  const int kind = j < a.hq ? 0 : (j < a.hq + a.hkv ? 1 : 2);  // q, k, v
  const int h = kind == 0 ? j : (kind == 1 ? j - a.hq : j - a.hq - a.hkv);
  const T* src;
  int64_t src_st;
  if (kind == 0) {
    src = reinterpret_cast<const T*>(a.q_in) + bi * a.qi_sb + (int64_t)h * a.qi_sh;
    src_st = a.qi_st;
  } else if (kind == 1) {
    src = reinterpret_cast<const T*>(a.k_in) + bi * a.ki_sb + (int64_t)h * a.ki_sh;
    src_st = a.ki_st;
  } else {
    src = reinterpret_cast<const T*>(a.v_in) + bi * a.vi_sb + (int64_t)h * a.vi_sh;
    src_st = a.vi_st;
  }
  src += E * sub + (int64_t)o_b * src_st;

  // the first pass's rows go out before the barrier
  RawE<T, E> xr[kTok];
  if (active) {
#pragma unroll
    for (int i = 0; i < kTok; ++i)
      if (t0 + i < t_end) xr[i] = load_raw<T, E, VEC>(src + (int64_t)(t0 + i) * src_st);
  }
  // The block's tokens fall into at most two pages when the block size is at
  // least the token tile: their block-table entries are read here, once and
  // early (their latency overlaps the row loads and the cos / sin staging),
  // instead of one dependent table read per token before its store.
  const int32_t start = a.start_pos[b];
  const int64_t row = a.row_ids ? (int64_t)a.row_ids[b] : b;
  const int32_t* bt = a.block_tables + row * a.bt_stride;
  int32_t lb_first = 0, lb_last = -1;
  int64_t ph_first = -1, ph_last = -1;
  if (active && kind != 0) {
    const int32_t p0 = start + t0, p1 = start + t_end - 1;
    if (p0 >= 0) {
      lb_first = a.bs_shift >= 0 ? (p0 >> a.bs_shift) : p0 / a.bs;
      lb_last = a.bs_shift >= 0 ? (p1 >> a.bs_shift) : p1 / a.bs;
      if (lb_last - lb_first <= 1) {
        if (lb_first < a.bt_width) ph_first = bt[lb_first];
        if (lb_last != lb_first && lb_last < a.bt_width) ph_last = bt[lb_last];
      } else {
        lb_last = -1;  // more than two pages: per-token reads below
      }
    }
  }
  // cos / sin rows of the block's tokens into shared memory
  {
    const int n = (t_end - t0) * D;
    const T* cs0 = reinterpret_cast<const T*>(a.cos) + bi * a.rope_sb + ((int64_t)o_b + t0) * a.rope_st;
    const T* sn0 = reinterpret_cast<const T*>(a.sin) + bi * a.rope_sb + ((int64_t)o_b + t0) * a.rope_st;
    for (int i = threadIdx.x; i < n; i += kWarps * 32) {
      const int tr = i / D, d = i - (i / D) * D;
      s_rope[0][tr][d] = cs0[(int64_t)tr * a.rope_st + d];
      s_rope[1][tr][d] = sn0[(int64_t)tr * a.rope_st + d];
    }
  }
  __syncthreads();
  if (!active) return;

  float w[E];
  if (kind == 2) {
#pragma unroll
    for (int e = 0; e < E; ++e) w[e] = 0.f;
  } else {
    load_e<T, E, VEC>(reinterpret_cast<const T*>(kind == 0 ? a.qw : a.kw) + E * sub, w);
  }
  T* qo = reinterpret_cast<T*>(a.q_out) + bi * a.qo_sb + (int64_t)h * a.qo_sh + E * sub;
  T* pool = reinterpret_cast<T*>(kind == 1 ? a.k_pool : a.v_pool);

  for (int tt = t0; tt < t_end; tt += kTok) {
    if (tt != t0) {
#pragma unroll
      for (int i = 0; i < kTok; ++i)
        if (tt + i < t_end) xr[i] = load_raw<T, E, VEC>(src + (int64_t)(tt + i) * src_st);
    }
#pragma unroll
    for (int i = 0; i < kTok; ++i) {
      const int t = tt + i;
      if (t >= t_end) break;
      constexpr int W = E * (int)sizeof(T) / 4;  // 32-bit words per lane
      uint32_t xw[W];
      if constexpr (std::is_same_v<T, __nv_bfloat16>) {
        raw_words<T, E>(xr[i], xw);
        if (kind != 2) {
          uint32_t cw[W], sw[W];
          raw_words<T, E>(*reinterpret_cast<const RawE<T, E>*>(&s_rope[0][t - t0][E * sub]), cw);
          raw_words<T, E>(*reinterpret_cast<const RawE<T, E>*>(&s_rope[1][t - t0][E * sub]), sw);
          norm_rope_bf16<E>(xw, w, cw, sw, a.eps, sub, hmask);
        }
      } else {
        float x[E];
        raw_to_f32<T, E>(xr[i], x);
        if (kind != 2) {
          float cs[E], sn[E];
          raw_to_f32<T, E>(*reinterpret_cast<const RawE<T, E>*>(&s_rope[0][t - t0][E * sub]), cs);
          raw_to_f32<T, E>(*reinterpret_cast<const RawE<T, E>*>(&s_rope[1][t - t0][E * sub]), sn);
          norm_rope<T, E>(x, w, cs, sn, a.eps, sub, hmask);
        }
        RawE<T, E> r;
        T* e = reinterpret_cast<T*>(&r);
#pragma unroll
        for (int k = 0; k < E; ++k) e[k] = from_f32<T>(x[k]);
        raw_words<T, E>(r, xw);
      }
      const int64_t tok = (int64_t)o_b + t;
      if (kind == 0) {
        store_words<T, E, VEC>(qo + tok * a.qo_st, xw);
        continue;
      }
      const int32_t pos = start + t;
      const int32_t lb = a.bs_shift >= 0 ? (pos >> a.bs_shift) : pos / a.bs;
      if (pos < 0 || lb >= a.bt_width) {
        if (sub == 0) raise_dev(a.err, BL_DEVERR_TABLE);
        continue;
      }
      const int64_t phys = lb == lb_first && lb_last >= 0 ? ph_first : (lb == lb_last ? ph_last : bt[lb]);
      if (phys < 0 || phys >= a.num_blocks) {
        if (sub == 0) raise_dev(a.err, BL_DEVERR_BLOCK_ID);
        continue;
      }
      const int64_t off = (((a.layer * a.num_blocks + phys) * a.hkv + h) * a.bs + (pos - lb * a.bs)) * D;
      store_words<T, E, VEC>(pool + off + E * sub, xw);
    }
  }
}

template <typename T, int E>
int launch_e(const PrepArgs& k, bool vec, int batch, cudaStream_t s) {
  const int pairs = (k.hq + 2 * k.hkv + 1) / 2;
  const dim3 grid((unsigned)((k.max_new + kTokTile - 1) / kTokTile), (unsigned)batch,
                  (unsigned)((pairs + kWarps - 1) / kWarps));
  if (vec)
    qk_prep_kernel<T, E, true><<<grid, kWarps * 32, 0, s>>>(k);
  else
    qk_prep_kernel<T, E, false><<<grid, kWarps * 32, 0, s>>>(k);
  BL_CHECK_LAUNCH("qk_prep_kernel");
  return BL_OK;
}

template <typename T>
int launch(const PrepArgs& k, int64_t d, bool vec, int batch, cudaStream_t s) {
  switch (d) {
    case 64: return launch_e<T, 4>(k, vec, batch, s);
    case 128: return launch_e<T, 8>(k, vec, batch, s);
    default: return launch_e<T, 16>(k, vec, batch, s);
  }
}

}  // namespace
}  // namespace bl

using namespace bl;

extern "C" int bl_qk_norm_rope_append(const bl_qk_prep_args* args, void* stream) {
  BL_CHECK_ARG(args != nullptr, "bl_qk_norm_rope_append: args is null");
  const bl_qk_prep_args& a = *args;
  int rc = check_paged_layer(a.kv, "bl_qk_norm_rope_append");
  if (rc) return rc;
  const int64_t d = a.kv.head_dim;
  BL_CHECK_ARG(d == 64 || d == 128 || d == 256, "bl_qk_norm_rope_append: head_dim must be 64, 128 or 256");
  BL_CHECK_ARG(a.q_in && a.k_in && a.v_in && a.q_out && a.q_norm_weight && a.k_norm_weight && a.cos && a.sin &&
                   a.start_pos,
               "bl_qk_norm_rope_append: null pointer argument");
  BL_CHECK_ARG(a.batch > 0 && a.max_new_tokens > 0, "K/V sequence length must be greater than zero");
  BL_CHECK_ARG(a.batch <= 65535, "bl_qk_norm_rope_append: batch must be at most 65535");
  BL_CHECK_ARG(a.max_new_tokens <= INT32_MAX, "bl_qk_norm_rope_append: too many new tokens");
  BL_CHECK_ARG(a.num_q_heads > 0 && a.num_q_heads % a.kv.num_kv_heads == 0,
               "num_heads must divide evenly by num_kv_heads");
  PrepArgs k;
  k.q_in = a.q_in;
  k.qi_sb = a.q_in_stride_b;
  k.qi_sh = a.q_in_stride_h;
  k.qi_st = a.q_in_stride_t;
  k.k_in = a.k_in;
  k.ki_sb = a.k_in_stride_b;
  k.ki_sh = a.k_in_stride_h;
  k.ki_st = a.k_in_stride_t;
  k.v_in = a.v_in;
  k.vi_sb = a.v_in_stride_b;
  k.vi_sh = a.v_in_stride_h;
  k.vi_st = a.v_in_stride_t;
  k.q_out = a.q_out;
  k.qo_sb = a.q_out_stride_b;
  k.qo_sh = a.q_out_stride_h;
  k.qo_st = a.q_out_stride_t;
  k.qw = a.q_norm_weight;
  k.kw = a.k_norm_weight;
  k.cos = a.cos;
  k.sin = a.sin;
  k.rope_sb = a.rope_stride_b;
  k.rope_st = a.rope_stride_t;
  k.eps = a.eps;
  k.hq = (int32_t)a.num_q_heads;
  k.hkv = (int32_t)a.kv.num_kv_heads;
  k.k_pool = a.kv.k_pool;
  k.v_pool = a.kv.v_pool;
  k.num_blocks = a.kv.num_blocks;
  k.layer = a.kv.layer;
  k.bs = (int32_t)a.kv.block_size;
  k.bs_shift = -1;
  for (int sh = 0; sh < 31; ++sh)
    if ((int64_t)1 << sh == a.kv.block_size) k.bs_shift = sh;
  k.block_tables = a.kv.block_tables;
  k.bt_stride = a.kv.bt_stride;
  k.bt_width = (int32_t)std::min<int64_t>(a.kv.bt_width, INT32_MAX);
  k.row_ids = a.kv.row_ids;
  k.start_pos = a.start_pos;
  k.new_offsets = a.new_offsets;
  k.max_new = (int32_t)a.max_new_tokens;
  k.err = a.err;
  // one vector per lane when every base and stride is aligned to E elements
  const int64_t es = elem_size(a.kv.dtype);
  const uint64_t vb = (uint64_t)(d / 16 * es);
  bool vec = true;
  const void* bases[] = {a.q_in, a.k_in, a.v_in, a.q_out, a.kv.k_pool, a.kv.v_pool, a.q_norm_weight, a.k_norm_weight,
                         a.cos, a.sin};
  for (const void* p : bases) vec = vec && (uint64_t)(uintptr_t)p % vb == 0;
  for (int64_t st : std::initializer_list<int64_t>{a.q_in_stride_b, a.q_in_stride_h, a.q_in_stride_t, a.k_in_stride_b, a.k_in_stride_h,
                     a.k_in_stride_t, a.v_in_stride_b, a.v_in_stride_h, a.v_in_stride_t, a.q_out_stride_b,
                     a.q_out_stride_h, a.q_out_stride_t, a.rope_stride_b, a.rope_stride_t})
    vec = vec && (uint64_t)(st * es) % vb == 0;
  cudaStream_t s = (cudaStream_t)stream;
  const int batch = (int)a.batch;
  switch (a.kv.dtype) {
    case BL_F32: return launch<float>(k, d, vec, batch, s);
    case BL_F16: return launch<__half>(k, d, vec, batch, s);
    default: return launch<__nv_bfloat16>(k, d, vec, batch, s);
  }
}
