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
// Grid (ceil(heads / 8), tokens, batch): warp w of block x handles row
// (token blockIdx.y, head x * 8 + w, batch row blockIdx.z), so no index needs a
// division; lane l holds elements [E*l, E*l + E) with E = D / 32, so RoPE's
// partner element d +- D/2 sits in lane l ^ 16.  With VEC every lane moves its
// E elements as one vector (the caller checks the alignment of every base
// and stride).
// Roofline: HBM.  Bytes per token: (Hq + 2 Hkv) * D * E_in read,
// (Hq + 2 Hkv) * D * E written, plus one cos and one sin row.
#include "common.cuh"

namespace bl {
namespace {

constexpr int kWarps = 8;
constexpr int kMaxGridY = 65535;

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
template <> struct VecOf<32> { struct alignas(16) type { uint4 lo, hi; }; };

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

template <typename T, int E, bool VEC>
__global__ void __launch_bounds__(kWarps * 32) qk_prep_kernel(const PrepArgs a) {
  constexpr int D = 32 * E;
  const int lane = threadIdx.x & 31;
  const int j = blockIdx.x * kWarps + (threadIdx.x >> 5);  // head row: q heads, then k, then v
  if (j >= a.hq + 2 * a.hkv) return;
  const int b = blockIdx.z;
  int n_b = a.max_new, o_b = 0;
  if (a.new_offsets) {
    o_b = a.new_offsets[b];
    n_b = a.new_offsets[b + 1] - o_b;
  }
  const int64_t bi = a.new_offsets ? 0 : b;  // packed inputs have one batch row
  const bool is_q = j < a.hq, is_k = !is_q && j < a.hq + a.hkv;
  const int h = is_q ? j : (is_k ? j - a.hq : j - a.hq - a.hkv);
  const T* src0;
  int64_t src_st;
  if (is_q) {
    src0 = reinterpret_cast<const T*>(a.q_in) + bi * a.qi_sb + (int64_t)h * a.qi_sh;
    src_st = a.qi_st;
  } else if (is_k) {
    src0 = reinterpret_cast<const T*>(a.k_in) + bi * a.ki_sb + (int64_t)h * a.ki_sh;
    src_st = a.ki_st;
  } else {
    src0 = reinterpret_cast<const T*>(a.v_in) + bi * a.vi_sb + (int64_t)h * a.vi_sh;
    src_st = a.vi_st;
  }
  float w[E];
  if (!is_q && !is_k) {
#pragma unroll
    for (int e = 0; e < E; ++e) w[e] = 0.f;
  } else {
    load_e<T, E, VEC>(reinterpret_cast<const T*>(is_q ? a.qw : a.kw) + E * lane, w);
  }
  const int64_t row = a.row_ids ? (int64_t)a.row_ids[b] : b;
  const int32_t start = a.start_pos[b];

  for (int t = blockIdx.y; t < n_b; t += gridDim.y) {
    const int64_t tok = (int64_t)o_b + t;  // index on the input T axis
    float x[E];
    load_e<T, E, VEC>(src0 + tok * src_st + E * lane, x);
    if (is_q || is_k) {
      // RMSNorm: fp32 mean square, rsqrt, weight, one rounding to T
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) ss = __fadd_rn(ss, __fmul_rn(x[e], x[e]));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
      const float rs = rsqrtf(__fadd_rn(ss / (float)D, a.eps));
#pragma unroll
      for (int e = 0; e < E; ++e) x[e] = round_to<T>(__fmul_rn(__fmul_rn(x[e], rs), w[e]));
      // RoPE (half-split): out = round(round(x * cos) + round(rotate_half(x) * sin))
      float cs[E], sn[E];
      const int64_t ro = bi * a.rope_sb + tok * a.rope_st + E * lane;
      load_e<T, E, VEC>(reinterpret_cast<const T*>(a.cos) + ro, cs);
      load_e<T, E, VEC>(reinterpret_cast<const T*>(a.sin) + ro, sn);
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const float partner = __shfl_xor_sync(0xffffffffu, x[e], 16);
        const float rot = lane < 16 ? -partner : partner;
        x[e] = round_to<T>(__fadd_rn(round_to<T>(__fmul_rn(x[e], cs[e])), round_to<T>(__fmul_rn(rot, sn[e]))));
      }
    }
    T* dst;
    if (is_q) {
      dst = reinterpret_cast<T*>(a.q_out) + bi * a.qo_sb + (int64_t)h * a.qo_sh + tok * a.qo_st;  // q_in's layout
    } else {
      const int32_t pos = start + t;
      const int32_t lb = a.bs_shift >= 0 ? (pos >> a.bs_shift) : pos / a.bs;
      if (pos < 0 || lb >= a.bt_width) {
        if (lane == 0) raise_dev(a.err, BL_DEVERR_TABLE);
        continue;
      }
      const int64_t phys = a.block_tables[row * a.bt_stride + lb];
      if (phys < 0 || phys >= a.num_blocks) {
        if (lane == 0) raise_dev(a.err, BL_DEVERR_BLOCK_ID);
        continue;
      }
      const int64_t off = ((a.layer * a.num_blocks + phys) * a.hkv + h) * a.bs + (pos - lb * a.bs);
      dst = reinterpret_cast<T*>(is_k ? a.k_pool : a.v_pool) + off * D;
    }
    store_e<T, E, VEC>(dst + E * lane, x);
  }
}

template <typename T, int E>
int launch_e(const PrepArgs& k, bool vec, int batch, cudaStream_t s) {
  const dim3 grid((unsigned)((k.hq + 2 * k.hkv + kWarps - 1) / kWarps), (unsigned)std::min(k.max_new, kMaxGridY),
                  (unsigned)batch);
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
    case 64: return launch_e<T, 2>(k, vec, batch, s);
    case 128: return launch_e<T, 4>(k, vec, batch, s);
    default: return launch_e<T, 8>(k, vec, batch, s);
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
  BL_CHECK_ARG(a.num_q_heads + 2 * a.kv.num_kv_heads <= 65535 * kWarps, "bl_qk_norm_rope_append: too many heads");
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
  const uint64_t vb = (uint64_t)(d / 32 * es);
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
