// Paged K/V append (slot-mapped scatter) and dense gather.
//
// Both are pure copies of head_dim-long rows between the caller's tensors and
// the paged pool [L, P, Hkv, bs, D].  They move each row with the widest
// vector (16/8/4/2 bytes) that divides the row and every base/stride, so at
// Qwen3 shapes (D=128, bf16: 256-byte rows) every thread moves 16 bytes.
// Both are HBM-bound; their algorithmic traffic is read + write of the rows.
//
// Reference semantics:
//   append: PagedLayerKV.append_only, src/barellm/engine/paged_kv_cache.py:151-193
//     positions = arange(start, end); phys = block_table[pos // bs];
//     key_cache[layer, phys, :, pos % bs, :] = key[0].transpose(0, 1)
//   gather: PagedLayerKV.read, src/barellm/engine/paged_kv_cache.py:215-240, plus
//     BatchLayerKV._pad, src/barellm/engine/batched_kv_cache.py:80-95 (zero padding).
#include "common.cuh"

namespace bl {
namespace {

template <int VEC> struct VecT;
template <> struct VecT<16> { using type = uint4; };
template <> struct VecT<8> { using type = uint2; };
template <> struct VecT<4> { using type = uint32_t; };
template <> struct VecT<2> { using type = uint16_t; };

struct AppendKernelArgs {
  char* k_pool;
  char* v_pool;
  const char* k_new;
  const char* v_new;
  int64_t num_blocks, hkv, row_bytes, layer;
  int32_t bs, bs_shift;   // bs_shift >= 0 when bs is a power of two
  int64_t nsb, nsh, nst;  // strides of the new K tokens, in bytes
  int64_t vsb, vsh, vst;  // strides of the new V tokens, in bytes
  const int32_t* block_tables;
  int64_t bt_stride;
  int32_t bt_width;
  const int32_t* row_ids;
  const int32_t* start_pos;
  const int32_t* new_offsets;
  int32_t max_new;
  int32_t nvec;
  int32_t* err;
};

constexpr int kAppendTok = 2;  // tokens per thread: both rows' loads are in flight before the stores

// grid: (ceil(max_new / (kAppendTok * blockDim.y)), hkv, batch); block (bx, by)
// with bx = min(nvec, 256): threadIdx.x walks the 16-byte vectors of a row,
// threadIdx.y the tokens, so a warp moves whole consecutive rows and no index
// needs a division (block_size is a shift when it is a power of two).
template <int VEC>
__global__ void __launch_bounds__(256) paged_append_kernel(const AppendKernelArgs a) {
  pdl_trigger();  // a dependent launch (the decode plan) may start; it waits for this grid
  using V = typename VecT<VEC>::type;
  const int b = blockIdx.z;
  const int h = blockIdx.y;
  int o_b = 0, n_b = a.max_new;
  if (a.new_offsets) {
    o_b = a.new_offsets[b];
    n_b = a.new_offsets[b + 1] - o_b;
  }
  const int t0 = blockIdx.x * (kAppendTok * blockDim.y) + threadIdx.y;
  if (t0 >= n_b) return;
  const int64_t row = a.row_ids ? (int64_t)a.row_ids[b] : b;
  const int32_t start = a.start_pos[b];
  const char* ksrc = a.k_new + (int64_t)b * a.nsb + (int64_t)h * a.nsh;
  const char* vsrc = a.v_new + (int64_t)b * a.vsb + (int64_t)h * a.vsh;
  int64_t src_t[kAppendTok], dst[kAppendTok];
  bool ok[kAppendTok];
#pragma unroll
  for (int i = 0; i < kAppendTok; ++i) {
    const int t = t0 + i * blockDim.y;
    ok[i] = t < n_b;
    src_t[i] = (int64_t)(o_b + t);
    dst[i] = 0;
    if (!ok[i]) continue;
    const int32_t pos = start + t;
    const int32_t lb = a.bs_shift >= 0 ? (pos >> a.bs_shift) : pos / a.bs;
    if (pos < 0 || lb >= a.bt_width) {
      raise_dev(a.err, BL_DEVERR_TABLE);
      ok[i] = false;
      continue;
    }
    const int64_t phys = a.block_tables[row * a.bt_stride + lb];
    if (phys < 0 || phys >= a.num_blocks) {
      raise_dev(a.err, BL_DEVERR_BLOCK_ID);
      ok[i] = false;
      continue;
    }
    dst[i] = (((a.layer * a.num_blocks + phys) * a.hkv + h) * a.bs + (pos - lb * a.bs)) * a.row_bytes;
  }
  for (int v = threadIdx.x; v < a.nvec; v += blockDim.x) {
    V kv[kAppendTok], vv[kAppendTok];
#pragma unroll
    for (int i = 0; i < kAppendTok; ++i) {
      if (ok[i]) {
        kv[i] = *reinterpret_cast<const V*>(ksrc + src_t[i] * a.nst + (int64_t)v * VEC);
        vv[i] = *reinterpret_cast<const V*>(vsrc + src_t[i] * a.vst + (int64_t)v * VEC);
      }
    }
#pragma unroll
    for (int i = 0; i < kAppendTok; ++i) {
      if (ok[i]) {
        *reinterpret_cast<V*>(a.k_pool + dst[i] + (int64_t)v * VEC) = kv[i];
        *reinterpret_cast<V*>(a.v_pool + dst[i] + (int64_t)v * VEC) = vv[i];
      }
    }
  }
}

struct GatherKernelArgs {
  const char* k_pool;
  const char* v_pool;
  char* k_out;
  char* v_out;
  int64_t num_blocks, hkv, bs, row_bytes, layer;
  int64_t osb, osh, ost;  // bytes
  const int32_t* block_tables;
  int64_t bt_stride, bt_width;
  const int32_t* row_ids;
  const int32_t* seq_lens;
  int64_t max_len;
  int32_t nvec;
  int32_t zero_fill;
  int32_t* err;
};

template <int VEC>
__global__ void __launch_bounds__(256) paged_gather_kernel(const GatherKernelArgs a) {
  using V = typename VecT<VEC>::type;
  const int64_t b = blockIdx.y;
  const uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t nvec = (uint32_t)a.nvec;
  const uint32_t v = idx % nvec;
  const uint32_t rest = idx / nvec;
  const int64_t t = rest % (uint32_t)a.max_len;
  const int64_t h = rest / (uint32_t)a.max_len;
  if (h >= a.hkv) return;
  const int64_t dst = b * a.osb + h * a.osh + t * a.ost + (int64_t)v * VEC;
  const int64_t len = a.seq_lens[b];
  if (t >= len) {
    if (a.zero_fill) {
      V z;
      memset(&z, 0, sizeof(V));
      *reinterpret_cast<V*>(a.k_out + dst) = z;
      *reinterpret_cast<V*>(a.v_out + dst) = z;
    }
    return;
  }
  const int64_t lb = t / a.bs;
  const int64_t off = t - lb * a.bs;
  if (lb >= a.bt_width) {
    raise_dev(a.err, BL_DEVERR_TABLE);
    return;
  }
  const int64_t row = a.row_ids ? (int64_t)a.row_ids[b] : b;
  const int64_t phys = a.block_tables[row * a.bt_stride + lb];
  if (phys < 0 || phys >= a.num_blocks) {
    raise_dev(a.err, BL_DEVERR_BLOCK_ID);
    return;
  }
  const int64_t src = (((a.layer * a.num_blocks + phys) * a.hkv + h) * a.bs + off) * a.row_bytes + (int64_t)v * VEC;
  const V kv = *reinterpret_cast<const V*>(a.k_pool + src);
  const V vv = *reinterpret_cast<const V*>(a.v_pool + src);
  *reinterpret_cast<V*>(a.k_out + dst) = kv;
  *reinterpret_cast<V*>(a.v_out + dst) = vv;
}

// widest vector (bytes) dividing every value
int pick_vec(std::initializer_list<uint64_t> vals) {
  for (int vec : {16, 8, 4, 2}) {
    bool ok = true;
    for (uint64_t x : vals) ok = ok && (x % (uint64_t)vec == 0);
    if (ok) return vec;
  }
  return 0;
}

}  // namespace
}  // namespace bl

using namespace bl;

extern "C" int bl_paged_append(const bl_append_args* args, void* stream) {
  BL_CHECK_ARG(args != nullptr, "bl_paged_append: args is null");
  const bl_append_args& a = *args;
  int rc = check_paged_layer(a.kv, "bl_paged_append");
  if (rc) return rc;
  BL_CHECK_ARG(a.k_new && a.v_new && a.start_pos, "bl_paged_append: null input pointer");
  BL_CHECK_ARG(a.batch > 0 && a.batch <= 65535, "bl_paged_append: batch must be in [1, 65535]");
  BL_CHECK_ARG(a.max_new_tokens > 0, "K/V sequence length must be greater than zero");
  const int64_t es = elem_size(a.kv.dtype);
  const int64_t row_bytes = a.kv.head_dim * es;
  const int vec = pick_vec({(uint64_t)row_bytes, (uint64_t)a.kv.k_pool, (uint64_t)a.kv.v_pool,
                            (uint64_t)a.k_new, (uint64_t)a.v_new,
                            (uint64_t)(a.new_stride_b * es), (uint64_t)(a.new_stride_h * es),
                            (uint64_t)(a.new_stride_t * es), (uint64_t)(a.v_stride_b * es),
                            (uint64_t)(a.v_stride_h * es), (uint64_t)(a.v_stride_t * es)});
  BL_CHECK_ARG(vec > 0, "bl_paged_append: tensors must be at least 2-byte aligned");

  BL_CHECK_ARG(a.max_new_tokens <= INT32_MAX, "bl_paged_append: too many new tokens");
  BL_CHECK_ARG(a.kv.num_kv_heads <= 65535, "bl_paged_append: too many KV heads");

  AppendKernelArgs k;
  k.k_pool = (char*)a.kv.k_pool;
  k.v_pool = (char*)a.kv.v_pool;
  k.k_new = (const char*)a.k_new;
  k.v_new = (const char*)a.v_new;
  k.num_blocks = a.kv.num_blocks;
  k.hkv = a.kv.num_kv_heads;
  k.row_bytes = row_bytes;
  k.layer = a.kv.layer;
  k.bs = (int32_t)a.kv.block_size;
  k.bs_shift = -1;
  for (int sh = 0; sh < 31; ++sh)
    if ((int64_t)1 << sh == a.kv.block_size) k.bs_shift = sh;
  k.nsb = a.new_stride_b * es;
  k.nsh = a.new_stride_h * es;
  k.nst = a.new_stride_t * es;
  k.vsb = a.v_stride_b * es;
  k.vsh = a.v_stride_h * es;
  k.vst = a.v_stride_t * es;
  k.block_tables = a.kv.block_tables;
  k.bt_stride = a.kv.bt_stride;
  k.bt_width = (int32_t)std::min<int64_t>(a.kv.bt_width, INT32_MAX);
  k.row_ids = a.kv.row_ids;
  k.start_pos = a.start_pos;
  k.new_offsets = a.new_offsets;
  k.max_new = (int32_t)a.max_new_tokens;
  k.nvec = (int32_t)(row_bytes / vec);
  k.err = a.err;

  const int bx = std::min(k.nvec, 256);
  int by = 256 / bx;  // fewer token rows per block when a row brings few tokens (decode)
  const int64_t tok_rows = (a.max_new_tokens + kAppendTok - 1) / kAppendTok;
  while (by > 1 && by / 2 >= tok_rows) by /= 2;
  const int64_t gx = (a.max_new_tokens + kAppendTok * by - 1) / (kAppendTok * by);
  dim3 block((unsigned)bx, (unsigned)by);
  dim3 grid((unsigned)gx, (unsigned)a.kv.num_kv_heads, (unsigned)a.batch);
  cudaStream_t s = (cudaStream_t)stream;
  switch (vec) {
    case 16: paged_append_kernel<16><<<grid, block, 0, s>>>(k); break;
    case 8: paged_append_kernel<8><<<grid, block, 0, s>>>(k); break;
    case 4: paged_append_kernel<4><<<grid, block, 0, s>>>(k); break;
    default: paged_append_kernel<2><<<grid, block, 0, s>>>(k); break;
  }
  BL_CHECK_LAUNCH("bl_paged_append");
  return BL_OK;
}

extern "C" int bl_paged_gather(const bl_gather_args* args, void* stream) {
  BL_CHECK_ARG(args != nullptr, "bl_paged_gather: args is null");
  const bl_gather_args& a = *args;
  int rc = check_paged_layer(a.kv, "bl_paged_gather");
  if (rc) return rc;
  BL_CHECK_ARG(a.k_out && a.v_out && a.seq_lens, "bl_paged_gather: null pointer");
  BL_CHECK_ARG(a.batch > 0 && a.batch <= 65535, "bl_paged_gather: batch must be in [1, 65535]");
  BL_CHECK_ARG(a.max_len > 0, "KV cache is empty");
  const int64_t es = elem_size(a.kv.dtype);
  const int64_t row_bytes = a.kv.head_dim * es;
  const int vec = pick_vec({(uint64_t)row_bytes, (uint64_t)a.kv.k_pool, (uint64_t)a.kv.v_pool,
                            (uint64_t)a.k_out, (uint64_t)a.v_out, (uint64_t)(a.out_stride_b * es),
                            (uint64_t)(a.out_stride_h * es), (uint64_t)(a.out_stride_t * es)});
  BL_CHECK_ARG(vec > 0, "bl_paged_gather: tensors must be at least 2-byte aligned");

  GatherKernelArgs k;
  k.k_pool = (const char*)a.kv.k_pool;
  k.v_pool = (const char*)a.kv.v_pool;
  k.k_out = (char*)a.k_out;
  k.v_out = (char*)a.v_out;
  k.num_blocks = a.kv.num_blocks;
  k.hkv = a.kv.num_kv_heads;
  k.bs = a.kv.block_size;
  k.row_bytes = row_bytes;
  k.layer = a.kv.layer;
  k.osb = a.out_stride_b * es;
  k.osh = a.out_stride_h * es;
  k.ost = a.out_stride_t * es;
  k.block_tables = a.kv.block_tables;
  k.bt_stride = a.kv.bt_stride;
  k.bt_width = a.kv.bt_width;
  k.row_ids = a.kv.row_ids;
  k.seq_lens = a.seq_lens;
  k.max_len = a.max_len;
  k.nvec = (int32_t)(row_bytes / vec);
  k.zero_fill = a.zero_fill;
  k.err = a.err;

  const int64_t per_row = a.max_len * k.hkv * k.nvec;
  const int threads = 256;
  const int64_t gx = (per_row + threads - 1) / threads;
  BL_CHECK_ARG(gx * threads <= (int64_t)UINT32_MAX, "bl_paged_gather: max_len too large");
  dim3 grid((unsigned)gx, (unsigned)a.batch);
  cudaStream_t s = (cudaStream_t)stream;
  switch (vec) {
    case 16: paged_gather_kernel<16><<<grid, threads, 0, s>>>(k); break;
    case 8: paged_gather_kernel<8><<<grid, threads, 0, s>>>(k); break;
    case 4: paged_gather_kernel<4><<<grid, threads, 0, s>>>(k); break;
    default: paged_gather_kernel<2><<<grid, threads, 0, s>>>(k); break;
  }
  BL_CHECK_LAUNCH("bl_paged_gather");
  return BL_OK;
}
