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
// One warp per (token, head) row; lane l holds elements [E*l, E*l + E) with
// E = D / 32, so RoPE's partner element d +- D/2 sits in lane l ^ 16.
// Roofline: HBM / latency.  Bytes per token: (Hq + 2 Hkv) * D * E_in read,
// (Hq + 2 Hkv) * D * E written.
#include "common.cuh"

namespace bl {
namespace {

constexpr int kWarps = 8;

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
  int64_t num_blocks, bs, layer;
  const int32_t* block_tables;
  int64_t bt_stride, bt_width;
  const int32_t* row_ids;
  const int32_t* start_pos;
  const int32_t* new_offsets;
  int64_t batch, max_new;
  int32_t* err;
};

template <typename T>
__device__ __forceinline__ float round_to(float x) {
  return to_f32<T>(from_f32<T>(x));
}

template <typename T, int E>
__global__ void __launch_bounds__(kWarps * 32) qk_prep_kernel(const PrepArgs a) {
  constexpr int D = 32 * E;
  const int lane = threadIdx.x & 31;
  const int64_t heads = a.hq + 2 * a.hkv;
  const int64_t r = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (r >= a.batch * a.max_new * heads) return;
  const int64_t slot = r / heads;
  const int j = (int)(r - slot * heads);
  const int64_t b = slot / a.max_new;
  const int64_t t = slot - b * a.max_new;
  int64_t tok = t;  // index on the input T axis
  if (a.new_offsets) {
    const int64_t o0 = a.new_offsets[b];
    if (t >= (int64_t)a.new_offsets[b + 1] - o0) return;
    tok = o0 + t;
  }
  const int64_t bi = a.new_offsets ? 0 : b;  // packed inputs have one batch row

  const T* src;
  const T* w = nullptr;
  if (j < a.hq) {
    src = reinterpret_cast<const T*>(a.q_in) + bi * a.qi_sb + j * a.qi_sh + tok * a.qi_st;
    w = reinterpret_cast<const T*>(a.qw);
  } else if (j < a.hq + a.hkv) {
    src = reinterpret_cast<const T*>(a.k_in) + bi * a.ki_sb + (j - a.hq) * a.ki_sh + tok * a.ki_st;
    w = reinterpret_cast<const T*>(a.kw);
  } else {
    src = reinterpret_cast<const T*>(a.v_in) + bi * a.vi_sb + (j - a.hq - a.hkv) * a.vi_sh + tok * a.vi_st;
  }
  float x[E];
#pragma unroll
  for (int e = 0; e < E; ++e) x[e] = to_f32<T>(src[E * lane + e]);

  if (w) {
    // RMSNorm: fp32 mean square, rsqrt, weight, one rounding to T
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) ss = __fadd_rn(ss, __fmul_rn(x[e], x[e]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    const float rs = rsqrtf(__fadd_rn(ss / (float)D, a.eps));
#pragma unroll
    for (int e = 0; e < E; ++e) x[e] = round_to<T>(__fmul_rn(__fmul_rn(x[e], rs), to_f32<T>(w[E * lane + e])));
    // RoPE (half-split): out = round(round(x * cos) + round(rotate_half(x) * sin))
    const T* cs = reinterpret_cast<const T*>(a.cos) + bi * a.rope_sb + tok * a.rope_st;
    const T* sn = reinterpret_cast<const T*>(a.sin) + bi * a.rope_sb + tok * a.rope_st;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float partner = __shfl_xor_sync(0xffffffffu, x[e], 16);
      const float rot = lane < 16 ? -partner : partner;
      const float c = to_f32<T>(cs[E * lane + e]), s = to_f32<T>(sn[E * lane + e]);
      x[e] = round_to<T>(__fadd_rn(round_to<T>(__fmul_rn(x[e], c)), round_to<T>(__fmul_rn(rot, s))));
    }
  }

  T* dst;
  if (j < a.hq) {
    dst = reinterpret_cast<T*>(a.q_out) + bi * a.qo_sb + j * a.qo_sh + tok * a.qo_st;  // same layout as q_in
  } else {
    const int h = j < a.hq + a.hkv ? j - a.hq : j - a.hq - a.hkv;
    const int64_t pos = (int64_t)a.start_pos[b] + t;
    const int64_t lb = pos / a.bs;
    const int64_t row = a.row_ids ? (int64_t)a.row_ids[b] : b;
    if (pos < 0 || lb >= a.bt_width) {
      if (lane == 0) raise_dev(a.err, BL_DEVERR_TABLE);
      return;
    }
    const int64_t phys = a.block_tables[row * a.bt_stride + lb];
    if (phys < 0 || phys >= a.num_blocks) {
      if (lane == 0) raise_dev(a.err, BL_DEVERR_BLOCK_ID);
      return;
    }
    const int64_t off = ((a.layer * a.num_blocks + phys) * a.hkv + h) * a.bs + (pos - lb * a.bs);
    dst = reinterpret_cast<T*>(j < a.hq + a.hkv ? a.k_pool : a.v_pool) + off * D;
  }
#pragma unroll
  for (int e = 0; e < E; ++e) dst[E * lane + e] = from_f32<T>(x[e]);
}

template <typename T>
int launch(const PrepArgs& k, int64_t d, cudaStream_t s) {
  const int64_t rows = k.batch * k.max_new * (k.hq + 2 * k.hkv);
  const unsigned grid = (unsigned)((rows + kWarps - 1) / kWarps);
  switch (d) {
    case 64: qk_prep_kernel<T, 2><<<grid, kWarps * 32, 0, s>>>(k); break;
    case 128: qk_prep_kernel<T, 4><<<grid, kWarps * 32, 0, s>>>(k); break;
    default: qk_prep_kernel<T, 8><<<grid, kWarps * 32, 0, s>>>(k); break;
  }
  BL_CHECK_LAUNCH("qk_prep_kernel");
  return BL_OK;
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
  BL_CHECK_ARG(a.num_q_heads > 0 && a.num_q_heads % a.kv.num_kv_heads == 0,
               "num_heads must divide evenly by num_kv_heads");
  const int64_t rows = a.batch * a.max_new_tokens * (a.num_q_heads + 2 * a.kv.num_kv_heads);
  BL_CHECK_ARG((rows + kWarps - 1) / kWarps <= INT32_MAX, "bl_qk_norm_rope_append: too many rows");
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
  k.bs = a.kv.block_size;
  k.layer = a.kv.layer;
  k.block_tables = a.kv.block_tables;
  k.bt_stride = a.kv.bt_stride;
  k.bt_width = a.kv.bt_width;
  k.row_ids = a.kv.row_ids;
  k.start_pos = a.start_pos;
  k.new_offsets = a.new_offsets;
  k.batch = a.batch;
  k.max_new = a.max_new_tokens;
  k.err = a.err;
  cudaStream_t s = (cudaStream_t)stream;
  switch (a.kv.dtype) {
    case BL_F32: return launch<float>(k, d, s);
    case BL_F16: return launch<__half>(k, d, s);
    default: return launch<__nv_bfloat16>(k, d, s);
  }
}
