// Cross-GPU plumbing of the KV-head-sharded decode: peer mapping of device
// memory between the processes of one node (CUDA IPC, plain peer mappings, no
// multicast objects) and the completion barrier that closes a call.
//
// Barrier protocol.  Every rank owns a signal pad of BL_MAX_RANKS int32 slots
// (slot s is written only by rank s) and a call counter `epoch`, all zero at
// the start.  Call k (epoch k) on rank r, after its attention and reduce
// kernels have stored their heads into every rank's gathered buffer:
//   lane i < world:  st.release.sys  pad_i[r] = k      ("my stores to you are done")
//                    spin ld.acquire.sys pad_r[i] until it reaches k
//                    (at most timeout_ns; then BL_DEVERR_TIMEOUT and return)
// The counters only grow, so a rank that is one call ahead can never be
// mistaken for the current one, and nothing is ever reset between calls --
// which also keeps the protocol valid inside a replayed CUDA graph.
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

#include "common.cuh"

namespace bl {
namespace {

constexpr int64_t kDefaultTimeoutNs = 2000000000LL;  // 2 s

struct PeerBarrierArgs {
  int32_t* pads[kMaxRanks];
  int32_t* epoch;
  int32_t world, rank;
  int64_t timeout_ns;
  int32_t* err;
};

template <typename P>
__device__ __forceinline__ P pick(const P (&arr)[kMaxRanks], int i) {
  P v = arr[0];
#pragma unroll
  for (int p = 1; p < kMaxRanks; ++p)
    if (p == i) v = arr[p];
  return v;
}

__global__ void __launch_bounds__(32) peer_barrier_kernel(const PeerBarrierArgs a) {
  const int i = threadIdx.x;
  const int32_t ep = *a.epoch + 1;
  if (i < a.world) {
    // The stores this rank made into the other ranks' buffers were issued by
    // kernels that completed before this one started; the fence orders them
    // before the release below at system scope.
    __threadfence_system();
    st_release_sys(pick(a.pads, i) + a.rank, ep);
    const int32_t* flag = pick(a.pads, a.rank) + i;
    const uint64_t t0 = global_timer_ns();
    while ((int32_t)((uint32_t)ld_acquire_sys(flag) - (uint32_t)ep) < 0) {
      if (global_timer_ns() - t0 > (uint64_t)a.timeout_ns) {
        raise_dev(a.err, BL_DEVERR_TIMEOUT);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncwarp();
  if (i == 0) *a.epoch = ep;
}

PFN_cuMemGetAddressRange_v3020 get_range_fn() {
  static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &p, 3020, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
  });
  return fn;
}

// CUDA IPC lets a process open a given allocation only once, and the
// exporter hands out the handle of the whole allocation (a caching-allocator
// segment can hold the regions of several objects).  So mappings are shared:
// one entry per distinct handle with a count of the addresses handed out from
// it, and the allocation is unmapped when the last of them is closed.
struct Mapping {
  unsigned char handle[sizeof(cudaIpcMemHandle_t)];
  void* base;
  int refs;
};
struct UserAddr {
  void* user;
  int mapping;  // index into g_maps
};
constexpr int kMaxMappings = 256;
std::mutex g_map_mu;
Mapping g_maps[kMaxMappings];
UserAddr g_users[kMaxMappings];
}  // namespace

int check_head_gather(const bl_head_gather& g, const char* who) {
  BL_CHECK_ARG(g.world >= 1 && g.world <= kMaxRanks, "%s: world must be in [1, %d], got %d", who, kMaxRanks,
               g.world);
  BL_CHECK_ARG(g.rank >= 0 && g.rank < g.world, "%s: rank %d outside [0, %d)", who, g.rank, g.world);
  BL_CHECK_ARG(g.head_offset >= 0, "%s: negative head_offset", who);
  BL_CHECK_ARG(g.epoch != nullptr, "%s: null epoch counter", who);
  for (int r = 0; r < g.world; ++r) {
    BL_CHECK_ARG(g.peer_out[r] != nullptr, "%s: null gathered buffer for rank %d", who, r);
    BL_CHECK_ARG(g.peer_signal[r] != nullptr, "%s: null signal pad for rank %d", who, r);
    BL_CHECK_ARG(((uintptr_t)g.peer_signal[r] & 3) == 0, "%s: signal pad of rank %d is not 4-byte aligned", who,
                 r);
  }
  return BL_OK;
}

int launch_peer_barrier(const bl_head_gather& g, int32_t* err, cudaStream_t s) {
  PeerBarrierArgs a = {};
  for (int r = 0; r < g.world; ++r) a.pads[r] = g.peer_signal[r];
  a.epoch = g.epoch;
  a.world = g.world;
  a.rank = g.rank;
  a.timeout_ns = g.timeout_ns > 0 ? g.timeout_ns : kDefaultTimeoutNs;
  a.err = err;
  peer_barrier_kernel<<<1, 32, 0, s>>>(a);
  BL_CHECK_LAUNCH("peer_barrier_kernel");
  return BL_OK;
}

}  // namespace bl

using namespace bl;

extern "C" int bl_ipc_export(const void* ptr, bl_ipc_handle* out) {
  BL_CHECK_ARG(ptr != nullptr && out != nullptr, "bl_ipc_export: null argument");
  auto range = get_range_fn();
  if (!range) {
    set_error("bl_ipc_export: cuMemGetAddressRange is unavailable from the driver");
    return BL_ERR_LAUNCH;
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  const CUresult r = range(&base, &size, (CUdeviceptr)(uintptr_t)ptr);
  if (r != CUDA_SUCCESS) {
    set_error("bl_ipc_export: cuMemGetAddressRange failed with CUresult %d (not device memory?)", (int)r);
    return BL_ERR_ARG;
  }
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, (void*)(uintptr_t)base);
  if (e != cudaSuccess) {
    set_error("bl_ipc_export: cudaIpcGetMemHandle failed: %s", cudaGetErrorString(e));
    return BL_ERR_LAUNCH;
  }
  static_assert(sizeof(h) <= sizeof(out->bytes), "IPC handle size");
  std::memset(out->bytes, 0, sizeof(out->bytes));
  std::memcpy(out->bytes, &h, sizeof(h));
  out->offset = (uint64_t)((uintptr_t)ptr - (uintptr_t)base);
  return BL_OK;
}

extern "C" int bl_ipc_import(const bl_ipc_handle* handle, void** ptr) {
  BL_CHECK_ARG(handle != nullptr && ptr != nullptr, "bl_ipc_import: null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle->bytes, sizeof(h));
  std::lock_guard<std::mutex> lk(g_map_mu);
  int slot = -1;
  for (int u = 0; u < kMaxMappings; ++u)
    if (g_users[u].user == nullptr) {
      slot = u;
      break;
    }
  if (slot < 0) {
    set_error("bl_ipc_import: more than %d imported addresses are open", kMaxMappings);
    return BL_ERR_CAPACITY;
  }
  int m = -1;
  for (int i = 0; i < kMaxMappings; ++i)
    if (g_maps[i].refs > 0 && std::memcmp(g_maps[i].handle, &h, sizeof(h)) == 0) {
      m = i;  // this allocation is mapped already: share the mapping
      break;
    }
  if (m < 0) {
    for (int i = 0; i < kMaxMappings; ++i)
      if (g_maps[i].refs == 0) {
        m = i;
        break;
      }
    // at most kMaxMappings user addresses exist, each holding one mapping, so a free entry remains
    void* base = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      set_error("bl_ipc_import: cudaIpcOpenMemHandle failed: %s", cudaGetErrorString(e));
      return BL_ERR_LAUNCH;
    }
    std::memcpy(g_maps[m].handle, &h, sizeof(h));
    g_maps[m].base = base;
    g_maps[m].refs = 0;
  }
  g_maps[m].refs += 1;
  void* user = (char*)g_maps[m].base + handle->offset;
  g_users[slot].user = user;
  g_users[slot].mapping = m;
  *ptr = user;
  return BL_OK;
}

extern "C" int bl_ipc_close(void* ptr) {
  BL_CHECK_ARG(ptr != nullptr, "bl_ipc_close: null pointer");
  void* unmap = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_map_mu);
    int slot = -1;
    for (int u = 0; u < kMaxMappings; ++u)
      if (g_users[u].user == ptr) {
        slot = u;
        break;
      }
    BL_CHECK_ARG(slot >= 0, "bl_ipc_close: address was not returned by bl_ipc_import (or is closed)");
    Mapping& m = g_maps[g_users[slot].mapping];
    g_users[slot].user = nullptr;
    if (--m.refs == 0) {
      unmap = m.base;
      m.base = nullptr;
      std::memset(m.handle, 0, sizeof(m.handle));
    }
  }
  if (unmap == nullptr) return BL_OK;  // other addresses still use this mapping
  const cudaError_t e = cudaIpcCloseMemHandle(unmap);
  if (e != cudaSuccess) {
    set_error("bl_ipc_close: cudaIpcCloseMemHandle failed: %s", cudaGetErrorString(e));
    return BL_ERR_LAUNCH;
  }
  return BL_OK;
}
