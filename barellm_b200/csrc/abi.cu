// Host-side plumbing of the C ABI: thread-local error text, shared argument
// checks, SM count cache and TMA descriptor creation through the driver
// entry point (no link-time dependency on libcuda).
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace bl {

static thread_local char g_last_error[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int check_paged_layer(const bl_paged_layer& kv, const char* who) {
  BL_CHECK_ARG(kv.k_pool && kv.v_pool, "%s: K/V pool pointers must be non-null", who);
  BL_CHECK_ARG(kv.num_layers > 0 && kv.num_blocks > 0 && kv.num_kv_heads > 0 &&
                   kv.block_size > 0 && kv.head_dim > 0,
               "%s: pool dimensions must be positive", who);
  BL_CHECK_ARG(kv.layer >= 0 && kv.layer < kv.num_layers, "%s: invalid layer index: %d", who,
               kv.layer);
  BL_CHECK_ARG(kv.num_blocks <= INT32_MAX, "%s: physical block id does not fit in int32 metadata",
               who);
  if (elem_size(kv.dtype) == 0) {
    set_error("%s: unsupported dtype code %d", who, kv.dtype);
    return BL_ERR_DTYPE;
  }
  BL_CHECK_ARG(kv.block_tables != nullptr, "%s: block_tables must be non-null", who);
  BL_CHECK_ARG(kv.bt_width > 0 && kv.bt_stride >= kv.bt_width,
               "%s: block table width/stride invalid (width %lld, stride %lld)", who,
               (long long)kv.bt_width, (long long)kv.bt_stride);
  return BL_OK;
}

int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (cached[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
  });
  return fn;
}

bool make_tmap_2d_16bit(CUtensorMap* map, const void* base, uint64_t row_elems, uint64_t rows,
                        uint32_t box_x, uint32_t box_y, bool bf16) {
  auto fn = get_encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is unavailable from the driver");
    return false;
  }
  cuuint64_t dims[2] = {row_elems, rows};
  cuuint64_t strides[1] = {row_elems * 2};
  cuuint32_t box[2] = {box_x, box_y};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                  const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed with CUresult %d", (int)r);
    return false;
  }
  return true;
}

// Paged pools viewed page by page: x = 64 elements (one 128-byte half of a
// 256-byte token row), y = 8 token rows (256 B apart), z = the row's two
// halves (128 B apart), w = groups of 8 rows (2 KB apart).  A box of
// {64, 8, 2, 2} is one whole 16-token page (4 KB), landing in shared memory as
// [8-row group][half][8 rows][128 B]: each 1 KB block is one 128-byte-swizzle
// atom, so a tile of pages is a K-major (or MN-major) tcgen05 operand with an
// 8-row group stride of 2 KB and the two halves 1 KB apart.
bool make_tmap_pages_16bit(CUtensorMap* map, const void* base, uint64_t rows, bool bf16) {
  auto fn = get_encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is unavailable from the driver");
    return false;
  }
  if (rows % 8 != 0) {
    set_error("page tensor map: %llu pool rows is not a multiple of 8", (unsigned long long)rows);
    return false;
  }
  cuuint64_t dims[4] = {64, 8, 2, rows / 8};
  cuuint64_t strides[3] = {256, 128, 2048};
  cuuint32_t box[4] = {64, 8, 2, 2};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled (page map) failed with CUresult %d", (int)r);
    return false;
  }
  return true;
}

namespace {
struct TmapEntry {
  const void* ptr;
  uint64_t rows;
  int dtype;
  int device;
  int kind;  // 0: rows (64 x 16 boxes), 1: whole pages
  CUtensorMap map;
};
std::mutex g_tmap_mu;
TmapEntry g_tmaps[32];
int g_tmap_next = 0;
}  // namespace

static bool get_cached_tmap(const void* pool, uint64_t rows, int dtype, int kind, CUtensorMap* out) {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(g_tmap_mu);
  for (auto& e : g_tmaps)
    if (e.ptr == pool && e.rows == rows && e.dtype == dtype && e.device == dev && e.kind == kind) {
      *out = e.map;
      return true;
    }
  TmapEntry& e = g_tmaps[g_tmap_next];
  const bool ok = kind == 0 ? make_tmap_2d_16bit(&e.map, pool, 128, rows, 64, 16, dtype == BL_BF16)
                            : make_tmap_pages_16bit(&e.map, pool, rows, dtype == BL_BF16);
  if (!ok) {
    e.ptr = nullptr;
    return false;
  }
  e.ptr = pool;
  e.rows = rows;
  e.dtype = dtype;
  e.device = dev;
  e.kind = kind;
  g_tmap_next = (g_tmap_next + 1) % 32;
  *out = e.map;
  return true;
}

bool get_pool_tmap(const void* pool, uint64_t rows, int dtype, CUtensorMap* out) {
  return get_cached_tmap(pool, rows, dtype, 0, out);
}

bool get_pool_page_tmap(const void* pool, uint64_t rows, int dtype, CUtensorMap* out) {
  return get_cached_tmap(pool, rows, dtype, 1, out);
}

}  // namespace bl

extern "C" {

const char* bl_last_error(void) { return bl::g_last_error; }

int bl_abi_version(void) { return BL_ABI_VERSION; }

}  // extern "C"
