// Paged (chunked) prefill attention, read in place.
//
// Query i of row b (C_b queries, total length L_b after the append) attends
// keys 0 .. L_b - C_b + i: the causal mask aligned to the bottom-right corner.
// With an empty prefix (L_b == C_b) this is exactly the reference prefill,
// SDPA(is_causal=True) at src/barellm/attention/backend.py:52-61; with a
// prefix it is chunked prefill, which the reference lists as future work
// (docs/ROADMAP.md:131) and whose oracle is gather + repeat + SDPA with an
// explicit bottom-right boolean mask.
//
// Kernels
//   prefill_simt_kernel   any dtype / head_dim <= 256 / block size / group:
//                         one CTA per (row, query, q-head).
//   prefill_tc_kernel     (prefill_tc.cu) bf16/fp16 tensor-core path.
#include <cstdlib>

#include "common.cuh"
#include "prefill_tc.cuh"

namespace bl {
namespace {

constexpr int kWarps = 4;
constexpr int kMaxDPL = 8;

struct SimtArgs {
  const void* q;
  int64_t q_sb, q_st, q_sh;
  void* out;
  int64_t o_sb, o_st, o_sh;
  const int32_t* q_offsets;
  const int32_t* seq_lens;
  const void* k_pool;
  const void* v_pool;
  int64_t num_blocks, hkv, bs, d, layer;
  const int32_t* block_tables;
  int64_t bt_stride, bt_width;
  const int32_t* row_ids;
  int32_t g;
  int64_t max_q;
  float scale;
  int32_t* err;
};

// grid: (max_q_len, hq, batch)
template <typename T>
__global__ void __launch_bounds__(kWarps * 32) prefill_simt_kernel(const SimtArgs a) {
  __shared__ float s_o[kWarps][kMaxDPL * 32];
  __shared__ float s_m[kWarps], s_l[kWarps];
  const int64_t i = blockIdx.x;
  const int hq = blockIdx.y;
  const int64_t b = blockIdx.z;
  int64_t qo = 0, nq = a.max_q;
  if (a.q_offsets) {
    qo = a.q_offsets[b];
    nq = (int64_t)a.q_offsets[b + 1] - qo;
  }
  if (i >= nq) return;
  const int64_t len = a.seq_lens[b];
  const int64_t last_key = len - nq + i;  // inclusive
  const int h = hq / a.g;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = a.row_ids ? (int64_t)a.row_ids[b] : b;
  const T* qp = reinterpret_cast<const T*>(a.q) + b * a.q_sb + (qo + i) * a.q_st + (int64_t)hq * a.q_sh;
  float qv[kMaxDPL], ov[kMaxDPL];
#pragma unroll
  for (int k = 0; k < kMaxDPL; ++k) {
    const int d = lane + 32 * k;
    qv[k] = d < a.d ? to_f32<T>(qp[d]) : 0.f;
    ov[k] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  const T* kp = reinterpret_cast<const T*>(a.k_pool);
  const T* vp = reinterpret_cast<const T*>(a.v_pool);
  for (int64_t t = warp; t <= last_key; t += kWarps) {
    const int64_t lb = t / a.bs;
    const int64_t off = t - lb * a.bs;
    if (lb >= a.bt_width) {
      raise_dev(a.err, BL_DEVERR_TABLE);
      break;
    }
    const int64_t phys = a.block_tables[row * a.bt_stride + lb];
    if (phys < 0 || phys >= a.num_blocks) {
      raise_dev(a.err, BL_DEVERR_BLOCK_ID);
      continue;
    }
    const int64_t base = (((a.layer * a.num_blocks + phys) * a.hkv + h) * a.bs + off) * a.d;
    float dot = 0.f;
#pragma unroll
    for (int k = 0; k < kMaxDPL; ++k) {
      const int d = lane + 32 * k;
      if (d < a.d) dot += qv[k] * to_f32<T>(kp[base + d]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    const float s = dot * a.scale;
    const float mn = fmaxf(m, s);
    const float al = expf(m - mn);
    const float p = expf(s - mn);
    l = l * al + p;
#pragma unroll
    for (int k = 0; k < kMaxDPL; ++k) {
      const int d = lane + 32 * k;
      ov[k] = ov[k] * al + (d < a.d ? p * to_f32<T>(vp[base + d]) : 0.f);
    }
    m = mn;
  }
#pragma unroll
  for (int k = 0; k < kMaxDPL; ++k) s_o[warp][lane + 32 * k] = ov[k];
  if (lane == 0) {
    s_m[warp] = m;
    s_l[warp] = l;
  }
  __syncthreads();
  float M = -INFINITY;
  for (int w = 0; w < kWarps; ++w) M = fmaxf(M, s_m[w]);
  T* op = reinterpret_cast<T*>(a.out) + b * a.o_sb + (qo + i) * a.o_st + (int64_t)hq * a.o_sh;
  for (int d = threadIdx.x; d < a.d; d += blockDim.x) {
    float L = 0.f, O = 0.f;
    for (int w = 0; w < kWarps; ++w) {
      const float f = (s_m[w] == -INFINITY) ? 0.f : expf(s_m[w] - M);
      L += f * s_l[w];
      O += f * s_o[w][d];
    }
    op[d] = from_f32<T>(L > 0.f ? O / L : 0.f);
  }
}

template <typename T>
int launch_simt(const bl_prefill_args& a, cudaStream_t s) {
  SimtArgs k;
  k.q = a.q;
  k.q_sb = a.q_stride_b;
  k.q_st = a.q_stride_t;
  k.q_sh = a.q_stride_h;
  k.out = a.out;
  k.o_sb = a.out_stride_b;
  k.o_st = a.out_stride_t;
  k.o_sh = a.out_stride_h;
  k.q_offsets = a.q_offsets;
  k.seq_lens = a.seq_lens;
  k.k_pool = a.kv.k_pool;
  k.v_pool = a.kv.v_pool;
  k.num_blocks = a.kv.num_blocks;
  k.hkv = a.kv.num_kv_heads;
  k.bs = a.kv.block_size;
  k.d = a.kv.head_dim;
  k.layer = a.kv.layer;
  k.block_tables = a.kv.block_tables;
  k.bt_stride = a.kv.bt_stride;
  k.bt_width = a.kv.bt_width;
  k.row_ids = a.kv.row_ids;
  k.g = (int32_t)(a.num_q_heads / a.kv.num_kv_heads);
  k.max_q = a.max_q_len;
  k.scale = a.scale;
  k.err = a.err;
  dim3 grid((unsigned)a.max_q_len, (unsigned)a.num_q_heads, (unsigned)a.batch);
  prefill_simt_kernel<T><<<grid, kWarps * 32, 0, s>>>(k);
  BL_CHECK_LAUNCH("prefill_simt_kernel");
  return BL_OK;
}

}  // namespace
}  // namespace bl

using namespace bl;

extern "C" int bl_prefill_path(int32_t dtype, int64_t head_dim, int64_t block_size, int64_t num_q_heads,
                               int64_t num_kv_heads) {
  return prefill_tc_supported(dtype, head_dim, block_size, num_q_heads, num_kv_heads) ? 1 : 0;
}

extern "C" int bl_paged_prefill(const bl_prefill_args* args, void* stream) {
  BL_CHECK_ARG(args != nullptr, "bl_paged_prefill: args is null");
  const bl_prefill_args& a = *args;
  int rc = check_paged_layer(a.kv, "bl_paged_prefill");
  if (rc) return rc;
  BL_CHECK_ARG(a.q && a.out && a.seq_lens, "bl_paged_prefill: null q/out/seq_lens");
  BL_CHECK_ARG(a.batch > 0 && a.batch <= 65535, "bl_paged_prefill: batch must be in [1, 65535]");
  BL_CHECK_ARG(a.num_q_heads > 0 && a.num_q_heads <= 65535 && a.num_q_heads % a.kv.num_kv_heads == 0,
               "num_heads must divide evenly by num_kv_heads");
  BL_CHECK_ARG(a.max_q_len > 0 && a.max_q_len <= INT32_MAX,
               "K/V sequence length must be greater than zero");
  BL_CHECK_ARG(a.kv.head_dim <= 256, "bl_paged_prefill: head_dim > 256 is not supported");
  cudaStream_t s = (cudaStream_t)stream;
  if (prefill_tc_supported(a.kv.dtype, a.kv.head_dim, a.kv.block_size, a.num_q_heads, a.kv.num_kv_heads))
    return prefill_tc_launch(a, s);
  switch (a.kv.dtype) {
    case BL_F32: return launch_simt<float>(a, s);
    case BL_F16: return launch_simt<__half>(a, s);
    default: return launch_simt<__nv_bfloat16>(a, s);
  }
}
