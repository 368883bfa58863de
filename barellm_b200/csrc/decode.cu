// Paged decode attention (one query token per request, GQA), read in place.
//
// Replaces, for the batched decode step, the reference chain
//   BatchLayerKV.read -> _pad -> repeat_interleave(G) -> attention_mask -> SDPA
// (src/barellm/attention/backend.py:34-61, src/barellm/engine/batched_kv_cache.py:65-102):
//   out[b, hq] = softmax_t(scale * q[b, hq] . K[b, hq / G, t]) @ V[b, hq / G, t],  t < len_b.
// No dense K/V copy is made: every (block, kv-head) page is read once, straight
// from the pool through the block table.
//
// Kernels
//   decode_plan_kernel      one CTA.  Splits every row into 512-token chunks
//                           ("units"; the count depends only on the row's own
//                           length) and writes the unit list, full chunks first
//                           and then partial chunks by decreasing size.
//   decode_tc_kernel        bf16/fp16, head_dim 128, block_size 16, G <= 8.
//                           Persistent CTAs walk (unit, kv-head) items.  One
//                           producer lane streams each 4 KiB K page and 4 KiB V
//                           page with 2-D TMA (128-byte swizzle) into an 8-slot
//                           mbarrier ring; 4 consumer warps each take every 4th
//                           page.  S^T = K Q^T and O^T += V^T P^T run on
//                           mma.sync m16n8k16 (tokens / dims in M, the GQA
//                           group in N), with the online softmax in fp32 and P
//                           transposed in registers by movmatrix.  Warps merge
//                           through shared memory; single-chunk rows write the
//                           output, others write (o, lse) partials.
//   decode_reduce_kernel    merges the partials of multi-chunk rows.
// The plan, attention and reduce kernels are launched with programmatic
// dependent launch: each may start while its predecessor finishes and waits
// (griddepcontrol.wait) before reading that predecessor's output.  (Merging
// split rows inside the attention kernel, by the CTA that finishes a row's
// last chunk, measured slower: the merge and its fences stall that CTA's page
// pipeline.)
//   decode_simt_kernel      any dtype / head_dim <= 256 / block_size / group:
//                           one CTA per (row, q-head), no split.
// Every kernel that writes the output stores each element through a short
// list of targets: the caller's buffer, or -- for the KV-head-sharded decode
// (bl_paged_decode_allgather, bottom of this file) -- every rank's gathered
// buffer in peer memory, so the all-gather rides on the epilogue's stores.
// Roofline: HBM.  Algorithmic bytes per launch = sum_b len_b * Hkv * D * 2 * E
// (K and V) + 2 * B * Hq * D * E (q, out).
#include <mutex>

#include "common.cuh"

namespace bl {
namespace {

constexpr int kChunkTokens = 512;  // split-K chunk; fixed so results are batch-invariant
// The plan kernel stamps its header with this value and the batch size; the
// attention kernel runs a plan only when both match, so a workspace that holds
// no plan (or another batch's) yields an error word, not stray reads.
constexpr int32_t kPlanMagic = 0x4e414c50;

// ---------------------------------------------------------------------------
// workspace layout
// ---------------------------------------------------------------------------
struct WsLayout {
  size_t hdr, row_base, exec, lse, o, total;
  int64_t max_units;
};

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

WsLayout ws_layout(int64_t batch, int64_t hq, int64_t d, int64_t bs, int64_t max_seq_len) {
  WsLayout w;
  const int64_t chunk_blocks = std::max<int64_t>(1, kChunkTokens / bs);
  const int64_t max_blocks = (max_seq_len + bs - 1) / bs;
  const int64_t per_row = std::max<int64_t>(1, (max_blocks + chunk_blocks - 1) / chunk_blocks);
  w.max_units = batch * per_row;
  size_t off = 0;
  w.hdr = off;      off += align256(4 * sizeof(int32_t));
  w.row_base = off; off += align256((batch + 1) * sizeof(int32_t));
  w.exec = off;     off += align256(w.max_units * 2 * sizeof(int32_t));
  w.lse = off;      off += align256(w.max_units * hq * sizeof(float));
  w.o = off;        off += align256(w.max_units * hq * d * sizeof(float));
  w.total = off;
  return w;
}

// ---------------------------------------------------------------------------
// plan
// ---------------------------------------------------------------------------
constexpr int kPlanThreads = 1024;

__device__ __forceinline__ int block_excl_scan(int v, int* warp_tot, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_tot[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int t = warp_tot[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += y;
    }
    warp_tot[lane] = t;  // inclusive
  }
  __syncthreads();
  const int warp_excl = warp ? warp_tot[warp - 1] : 0;
  total = warp_tot[31];
  __syncthreads();
  return warp_excl + x - v;
}

struct PlanArgs {
  const int32_t* seq_lens;
  int32_t batch, bs, chunk_blocks, bt_width, max_units;
  int32_t* hdr;       // [0] total units
  int32_t* row_base;  // [batch + 1]
  int2* exec;         // [max_units] (row, chunk)
  int32_t* err;
};

__device__ __forceinline__ int row_blocks(int len, int bs, int bt_width, int32_t* err) {
  if (len <= 0) return 0;
  int nb = (len + bs - 1) / bs;
  if (nb > bt_width) {
    raise_dev(err, BL_DEVERR_TABLE);
    nb = bt_width;
  }
  return nb;
}

__global__ void __launch_bounds__(kPlanThreads) decode_plan_kernel(const PlanArgs a) {
  // the attention kernel may launch now; it waits for this grid (and, through
  // the pdl_wait below, for the append before it) before reading the plan
  pdl_trigger();
  __shared__ int warp_tot[32];
  __shared__ int hist[kChunkTokens + 1];    // partial-chunk sizes (blocks), 1..chunk_blocks-1
  __shared__ int bucket[kChunkTokens + 1];
  const int cb = a.chunk_blocks;
  for (int i = threadIdx.x; i <= cb; i += blockDim.x) hist[i] = 0;
  __syncthreads();

  // pass 1: row_base (all chunks) and the full-chunk positions
  int carry_all = 0, carry_full = 0;
  for (int base = 0; base < a.batch; base += blockDim.x) {
    const int b = base + threadIdx.x;
    int nb = 0;
    if (b < a.batch) nb = row_blocks(a.seq_lens[b], a.bs, a.bt_width, a.err);
    const int nch = (nb + cb - 1) / cb;
    const int nfull = nb / cb;
    int tot_all, tot_full;
    const int ex_all = block_excl_scan(nch, warp_tot, tot_all);
    const int ex_full = block_excl_scan(nfull, warp_tot, tot_full);
    if (b < a.batch) {
      a.row_base[b] = carry_all + ex_all;
      const int p0 = carry_full + ex_full;
      for (int c = 0; c < nfull; ++c)
        if (p0 + c < a.max_units) a.exec[p0 + c] = make_int2(b, c);
      const int rem = nb - nfull * cb;
      if (rem > 0) atomicAdd(&hist[rem], 1);
    }
    carry_all += tot_all;
    carry_full += tot_full;
  }
  if (threadIdx.x == 0) a.row_base[a.batch] = carry_all;
  __syncthreads();
  // bucket starts, largest partial size first
  if (threadIdx.x == 0) {
    int pos = carry_full;
    for (int s = cb - 1; s >= 1; --s) {
      bucket[s] = pos;
      pos += hist[s];
    }
    int total = carry_all;
    if (total > a.max_units) {
      raise_dev(a.err, BL_DEVERR_WORKSPACE);
      total = a.max_units;
    }
    a.hdr[0] = total;
    a.hdr[1] = kPlanMagic;
    a.hdr[2] = a.batch;
  }
  __syncthreads();
  // pass 2: scatter partial chunks into their size buckets
  for (int b = threadIdx.x; b < a.batch; b += blockDim.x) {
    const int nb = row_blocks(a.seq_lens[b], a.bs, a.bt_width, nullptr);
    const int nfull = nb / cb;
    const int rem = nb - nfull * cb;
    if (rem > 0) {
      const int p = atomicAdd(&bucket[rem], 1);
      if (p < a.max_units) a.exec[p] = make_int2(b, nfull);
    }
  }
  // complete only after the previous kernel (the step's K/V append) has
  pdl_wait();
}

// ---------------------------------------------------------------------------
// tensor-core decode kernel
// ---------------------------------------------------------------------------
constexpr int kD = 128;
constexpr int kBS = 16;
constexpr int kNW = 4;                        // consumer warps
constexpr int kThreadsTC = (kNW + 1) * 32;    // + one producer warp
constexpr int kStages = 8;
constexpr int kPageBytes = kBS * kD * 2;      // 4 KiB
constexpr int kSlotBytes = 2 * kPageBytes;    // K + V
constexpr float kLog2e = 1.4426950408889634f;

struct TCArgs {
  const void* q;
  int64_t q_sb, q_sh;
  OutTargets out;
  int64_t o_sb, o_sh;
  const int32_t* block_tables;
  int64_t bt_stride;
  int32_t bt_width;
  const int32_t* row_ids;
  const int32_t* seq_lens;
  int32_t batch, hq, hkv, g;
  int64_t num_blocks;
  int64_t layer_row0;  // layer * num_blocks * hkv * bs (pool row of block 0, head 0)
  float scale_log2;
  int32_t chunk_blocks;
  const int32_t* hdr;
  const int32_t* row_base;
  const int2* exec;
  float* ws_lse;
  float* ws_o;
  int32_t max_units;
  int32_t* err;
};

struct TCShared {
  // slots live at the (1024-aligned) start of dynamic smem; this struct follows
  uint64_t full[kStages];
  uint64_t empty[kStages];
  int abort;
};

// A plan unit (row, chunk) is used only when the row is in the batch and the
// chunk lies inside the row's current length; the producer and the consumers
// apply the same test, so they always agree on the pages of an item.
__device__ __forceinline__ bool unit_in_range(const TCArgs& a, int2 bc, int& len, int& nbt) {
  if (bc.x < 0 || bc.x >= a.batch || bc.y < 0) return false;
  len = a.seq_lens[bc.x];
  nbt = min((len + kBS - 1) / kBS, a.bt_width);
  return bc.y * a.chunk_blocks < nbt;
}

template <typename T>
__global__ void __launch_bounds__(kThreadsTC) decode_tc_kernel(const TCArgs a,
                                                               const __grid_constant__ CUtensorMap kmap,
                                                               const __grid_constant__ CUtensorMap vmap) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // 1024-byte alignment for the 128B-swizzled TMA tiles
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* slots = smem;
  float* comb_o = reinterpret_cast<float*>(smem + kStages * kSlotBytes);   // [kNW][g][kD]
  float* comb_ml = comb_o + kNW * a.g * kD;                                // [kNW][8][2]
  TCShared* sh = reinterpret_cast<TCShared*>(comb_ml + kNW * 8 * 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sh->full[s], 1);
      mbar_init(&sh->empty[s], 1);
    }
    sh->abort = 0;
    fence_mbar_init();
  }
  __syncthreads();

  pdl_wait();  // the plan (and the append before it) are complete and visible
  int units = a.hdr[0];
  if (a.hdr[1] != kPlanMagic || a.hdr[2] != a.batch || units < 0 || units > a.max_units) {
    if (threadIdx.x == 0 && blockIdx.x == 0) raise_dev(a.err, BL_DEVERR_WORKSPACE);
    units = 0;
  }
  const int total_items = units * a.hkv;
  const int cb = a.chunk_blocks;

  if (warp == kNW) {
    // ------------------------------ producer ------------------------------
    if (lane != 0) return;
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
    const uint64_t policy = policy_evict_first();
    int issued = 0;  // pages issued so far == ring index of the next page
    bool ok = true;
    for (int item = blockIdx.x; item < total_items && ok; item += gridDim.x) {
      const int u = item / a.hkv;
      const int h = item - u * a.hkv;
      const int2 bc = a.exec[u];
      int len, nbt;
      if (!unit_in_range(a, bc, len, nbt)) {
        raise_dev(a.err, BL_DEVERR_WORKSPACE);
        continue;
      }
      const int lb0 = bc.y * cb;
      const int nb = min(cb, nbt - lb0);
      const int64_t row = a.row_ids ? (int64_t)a.row_ids[bc.x] : (int64_t)bc.x;
      const int32_t* bt = a.block_tables + row * a.bt_stride + lb0;
      for (int i = 0; i < nb; ++i) {
        const int gi = issued;
        const int slot = gi % kStages;
        if (!mbar_wait(&sh->empty[slot], ((gi / kStages) & 1) ^ 1)) {
          raise_dev(a.err, BL_DEVERR_TIMEOUT);
          sh->abort = 1;
          ok = false;
          break;
        }
        int64_t phys = bt[i];
        if (phys < 0 || phys >= a.num_blocks) {
          raise_dev(a.err, BL_DEVERR_BLOCK_ID);
          phys = 0;
        }
        const int32_t y = (int32_t)(a.layer_row0 + (phys * a.hkv + h) * kBS);
        unsigned char* dst = slots + slot * kSlotBytes;
        mbar_arrive_expect_tx(&sh->full[slot], kSlotBytes);
        tma_load_2d_hint(dst, &kmap, &sh->full[slot], 0, y, policy);
        tma_load_2d_hint(dst + kPageBytes / 2, &kmap, &sh->full[slot], 64, y, policy);
        tma_load_2d_hint(dst + kPageBytes, &vmap, &sh->full[slot], 0, y, policy);
        tma_load_2d_hint(dst + kPageBytes + kPageBytes / 2, &vmap, &sh->full[slot], 64, y, policy);
        ++issued;
      }
    }
    // Drain: wait (bounded) until every issued copy has landed, so no TMA
    // write can target this CTA's shared memory after it exits.
    for (int s = 0; s < kStages && s < issued; ++s) {
      const int last = s + ((issued - 1 - s) / kStages) * kStages;  // last page that used slot s
      if (!mbar_wait(&sh->full[s], (last / kStages) & 1)) raise_dev(a.err, BL_DEVERR_TIMEOUT);
    }
    return;
  }

  // ------------------------------ consumers ------------------------------
  const int g_row = lane >> 2;  // mma "groupID"
  const int t4 = lane & 3;      // thread in group
  const int tok_k = lane & 15;  // ldmatrix row for K (non-trans)
  const int hi_k = lane >> 4;
  const int tok_v = (lane & 7) + ((lane >> 4) << 3);
  const int hi_v = (lane >> 3) & 1;
  const T* qbase = reinterpret_cast<const T*>(a.q);
  int gblk = 0;

  for (int item = blockIdx.x; item < total_items; item += gridDim.x) {
    const int u = item / a.hkv;
    const int h = item - u * a.hkv;
    const int2 bc = a.exec[u];
    int len, nbt;
    if (!unit_in_range(a, bc, len, nbt)) continue;  // flagged by the producer
    const int b = bc.x;
    const int lb0 = bc.y * cb;
    const int nb = min(cb, nbt - lb0);
    const int nch = (nbt + cb - 1) / cb;

    // Q^T fragments (B operand, k = dim, n = head within the group)
    uint32_t qf[8][2];
    {
      const bool valid = g_row < a.g;
      const T* qp = qbase + (int64_t)b * a.q_sb + (int64_t)(h * a.g + (valid ? g_row : 0)) * a.q_sh;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        qf[ks][0] = valid ? *reinterpret_cast<const uint32_t*>(qp + ks * 16 + 2 * t4) : 0u;
        qf[ks][1] = valid ? *reinterpret_cast<const uint32_t*>(qp + ks * 16 + 8 + 2 * t4) : 0u;
      }
    }

    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    float o[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;

    for (int i = warp; i < nb; i += kNW) {
      const int gi = gblk + i;
      const int slot = gi % kStages;
      if (*(volatile int*)&sh->abort) break;
      if (!mbar_wait(&sh->full[slot], (gi / kStages) & 1)) {
        raise_dev(a.err, BL_DEVERR_TIMEOUT);
        *(volatile int*)&sh->abort = 1;
        break;
      }
      const uint32_t kb = smem_u32(slots + slot * kSlotBytes);
      const uint32_t vb = kb + kPageBytes;

      // S^T[token][head] = K[token] . q[head]
      float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const int cc = 2 * (ks & 3) + hi_k;
        const uint32_t addr = kb + (ks >> 2) * (kPageBytes / 2) + tok_k * 128 + ((cc ^ (tok_k & 7)) << 4);
        uint32_t a0, a1, a2, a3;
        ldmatrix_x4(addr, a0, a1, a2, a3);
        mma_16816<T>(s0, s1, s2, s3, a0, a1, a2, a3, qf[ks][0], qf[ks][1]);
      }
      // online softmax over tokens (rows), per head (column)
      const int pos0 = (lb0 + i) * kBS + g_row;
      float x0 = s0 * a.scale_log2, x1 = s1 * a.scale_log2;
      float x2 = s2 * a.scale_log2, x3 = s3 * a.scale_log2;
      if (pos0 >= len) x0 = x1 = -INFINITY;
      if (pos0 + 8 >= len) x2 = x3 = -INFINITY;
      float mx0 = fmaxf(x0, x2), mx1 = fmaxf(x1, x3);
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
      }
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      const float al0 = fast_exp2(m0 - mn0), al1 = fast_exp2(m1 - mn1);
      const float p0 = fast_exp2(x0 - mn0), p2 = fast_exp2(x2 - mn0);
      const float p1 = fast_exp2(x1 - mn1), p3 = fast_exp2(x3 - mn1);
      m0 = mn0;
      m1 = mn1;
      l0 = l0 * al0 + (p0 + p2);
      l1 = l1 * al1 + (p1 + p3);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        o[j][0] *= al0;
        o[j][2] *= al0;
        o[j][1] *= al1;
        o[j][3] *= al1;
      }
      // P^T (tokens x heads) -> B operand (k = token, n = head) via transpose
      const uint32_t pb0 = movmatrix_trans(pack2<T>(p0, p1));
      const uint32_t pb1 = movmatrix_trans(pack2<T>(p2, p3));
      // Pool slots past the row's length hold stale bytes (possibly NaN/Inf);
      // p is 0 there, but 0 * NaN is NaN, so those V elements are zeroed in
      // registers.  a0/a1 hold tokens 2*t4 + {0,1}, a2/a3 tokens 8 + 2*t4 + {0,1}.
      const int nvalid = len - (lb0 + i) * kBS;
      uint32_t vmask_lo = 0xffffffffu, vmask_hi = 0xffffffffu;
      if (nvalid < kBS) {
        vmask_lo = (2 * t4 < nvalid ? 0x0000ffffu : 0u) | (2 * t4 + 1 < nvalid ? 0xffff0000u : 0u);
        vmask_hi = (8 + 2 * t4 < nvalid ? 0x0000ffffu : 0u) | (9 + 2 * t4 < nvalid ? 0xffff0000u : 0u);
      }
      // O^T[dim][head] += V^T[dim][token] P^T[token][head]
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int cc = 2 * (j & 3) + hi_v;
        const uint32_t addr = vb + (j >> 2) * (kPageBytes / 2) + tok_v * 128 + ((cc ^ (tok_v & 7)) << 4);
        uint32_t a0, a1, a2, a3;
        ldmatrix_x4_trans(addr, a0, a1, a2, a3);
        mma_16816<T>(o[j][0], o[j][1], o[j][2], o[j][3], a0 & vmask_lo, a1 & vmask_lo, a2 & vmask_hi,
                     a3 & vmask_hi, pb0, pb1);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh->empty[slot]);
    }
    gblk += nb;

    // ---- merge the warps' partial softmax states ----
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, off);
      l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }
    const int h0 = 2 * t4, h1 = 2 * t4 + 1;
    if (g_row == 0) {
      comb_ml[(warp * 8 + h0) * 2 + 0] = m0;
      comb_ml[(warp * 8 + h0) * 2 + 1] = l0;
      comb_ml[(warp * 8 + h1) * 2 + 0] = m1;
      comb_ml[(warp * 8 + h1) * 2 + 1] = l1;
    }
    float* cw = comb_o + warp * a.g * kD;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int d0 = 16 * j + g_row;
      if (h0 < a.g) {
        cw[h0 * kD + d0] = o[j][0];
        cw[h0 * kD + d0 + 8] = o[j][2];
      }
      if (h1 < a.g) {
        cw[h1 * kD + d0] = o[j][1];
        cw[h1 * kD + d0 + 8] = o[j][3];
      }
    }
    named_barrier_sync(1, kNW * 32);
    const int ctid = threadIdx.x;  // 0 .. kNW*32-1
    if (nch <= 1 && a.out.vec16) {
      // a one-chunk row's output: eight consecutive dims per thread, one
      // 16-byte store per target
      for (int e = ctid; e < a.g * (kD / 8); e += kNW * 32) {
        const int hd = e / (kD / 8);
        const int d0 = (e - hd * (kD / 8)) * 8;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kNW; ++w) M = fmaxf(M, comb_ml[(w * 8 + hd) * 2]);
        float L = 0.f, O[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int w = 0; w < kNW; ++w) {
          const float mw = comb_ml[(w * 8 + hd) * 2];
          const float f = (mw == -INFINITY) ? 0.f : fast_exp2(mw - M);
          L += f * comb_ml[(w * 8 + hd) * 2 + 1];
          const float4* src = reinterpret_cast<const float4*>(comb_o + (w * a.g + hd) * kD + d0);
          const float4 u = src[0], v = src[1];
          O[0] += f * u.x, O[1] += f * u.y, O[2] += f * u.z, O[3] += f * u.w;
          O[4] += f * v.x, O[5] += f * v.y, O[6] += f * v.z, O[7] += f * v.w;
        }
        // the same arithmetic as the element-wise path below (O / L), so the
        // result does not depend on which store path runs
        float r[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) r[i] = (L > 0.f) ? O[i] / L : 0.f;
        uint4 pk;
        pk.x = pack2<T>(r[0], r[1]);
        pk.y = pack2<T>(r[2], r[3]);
        pk.z = pack2<T>(r[4], r[5]);
        pk.w = pack2<T>(r[6], r[7]);
        store_targets_x16b<T>(a.out, (int64_t)b * a.o_sb + (int64_t)(h * a.g + hd) * a.o_sh + d0, pk);
      }
      named_barrier_sync(1, kNW * 32);
      continue;
    }
    for (int e = ctid; e < a.g * kD; e += kNW * 32) {
      const int hd = e / kD;
      const int d = e - hd * kD;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kNW; ++w) M = fmaxf(M, comb_ml[(w * 8 + hd) * 2]);
      float L = 0.f, O = 0.f;
#pragma unroll
      for (int w = 0; w < kNW; ++w) {
        const float mw = comb_ml[(w * 8 + hd) * 2];
        const float f = (mw == -INFINITY) ? 0.f : fast_exp2(mw - M);
        L += f * comb_ml[(w * 8 + hd) * 2 + 1];
        O += f * comb_o[(w * a.g + hd) * kD + d];
      }
      const int hq = h * a.g + hd;
      const float val = (L > 0.f) ? O / L : 0.f;
      if (nch <= 1) {
        store_targets<T>(a.out, (int64_t)b * a.o_sb + (int64_t)hq * a.o_sh + d, from_f32<T>(val));
      } else {
        const int64_t slot_u = (int64_t)a.row_base[b] + bc.y;
        if (slot_u < 0 || slot_u >= a.max_units) continue;  // plan overflow, flagged by the plan kernel
        a.ws_o[(slot_u * a.hq + hq) * kD + d] = val;
        if (d == 0) a.ws_lse[slot_u * a.hq + hq] = (L > 0.f) ? M + __log2f(L) : -INFINITY;
      }
    }
    named_barrier_sync(1, kNW * 32);
  }
}

// ---------------------------------------------------------------------------
// split-K reduce
// ---------------------------------------------------------------------------
struct ReduceArgs {
  OutTargets out;
  int64_t o_sb, o_sh;
  const int32_t* seq_lens;
  int32_t bs, chunk_blocks, bt_width, hq, d;
  const int32_t* row_base;
  const float* ws_lse;
  const float* ws_o;
  int32_t max_units;
};

constexpr int kReduceMaxChunks = 1024;  // chunks whose weights the reduce keeps in shared memory

// grid (batch, hq); block = d threads
template <typename T>
__global__ void __launch_bounds__(256) decode_reduce_kernel(const ReduceArgs a) {
  pdl_wait();  // the attention kernel's partials are complete and visible
  const int b = blockIdx.x;
  const int hq = blockIdx.y;
  const int len = a.seq_lens[b];
  if (len <= 0) return;
  int nbt = (len + a.bs - 1) / a.bs;
  nbt = min(nbt, a.bt_width);
  const int nch = (nbt + a.chunk_blocks - 1) / a.chunk_blocks;
  if (nch <= 1) return;
  const int64_t base = a.row_base[b];
  if (base < 0 || base + nch > a.max_units) return;  // plan overflow, flagged by the plan kernel
  // blockDim.x == a.d == kD (four warps): one output element per thread
  __shared__ __align__(16) T s_out[kD];
  __shared__ float s_w[kReduceMaxChunks];
  __shared__ float s_red[kD / 32];
  const int d = threadIdx.x;
  float num = 0.f, den = 0.f;
  if (nch <= kReduceMaxChunks) {
    // The chunks' log-sum-exps are read once, by all threads at the same
    // time, and their weights kept in shared memory; each thread then sums its
    // dimension over the chunks with independent loads.  (Reading them chunk
    // by chunk in every thread made the reduce a chain of dependent global
    // loads.)  The arithmetic and its order are those of the plain loop below.
    float mloc = -INFINITY;
    for (int c = d; c < nch; c += kD) {
      const float l = a.ws_lse[(base + c) * a.hq + hq];
      s_w[c] = l;
      mloc = fmaxf(mloc, l);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, o));
    if ((d & 31) == 0) s_red[d >> 5] = mloc;
    __syncthreads();
    float M = s_red[0];
#pragma unroll
    for (int w = 1; w < kD / 32; ++w) M = fmaxf(M, s_red[w]);
    for (int c = d; c < nch; c += kD) {
      const float l = s_w[c];
      s_w[c] = (l == -INFINITY) ? 0.f : fast_exp2(l - M);
    }
    __syncthreads();
    const float* po = a.ws_o + (base * a.hq + hq) * a.d + d;
    const int64_t cstride = (int64_t)a.hq * a.d;
#pragma unroll 8
    for (int c = 0; c < nch; ++c) {
      const float w = s_w[c];
      num += w * po[c * cstride];
      den += w;
    }
  } else {
    float M = -INFINITY;
    for (int c = 0; c < nch; ++c) M = fmaxf(M, a.ws_lse[(base + c) * a.hq + hq]);
    for (int c = 0; c < nch; ++c) {
      const float lse = a.ws_lse[(base + c) * a.hq + hq];
      const float w = (lse == -INFINITY) ? 0.f : fast_exp2(lse - M);
      num += w * a.ws_o[((base + c) * a.hq + hq) * a.d + d];
      den += w;
    }
  }
  const T val = from_f32<T>(den > 0.f ? num / den : 0.f);
  const int64_t row = (int64_t)b * a.o_sb + (int64_t)hq * a.o_sh;
  if (!a.out.vec16) {
    store_targets<T>(a.out, row + d, val);
    return;
  }
  // the row leaves as 16-byte stores (one per eight elements and target)
  s_out[d] = val;
  __syncthreads();
  if (d < kD / 8) store_targets_x16b<T>(a.out, row + d * 8, reinterpret_cast<const uint4*>(s_out)[d]);
}

// ---------------------------------------------------------------------------
// generic SIMT decode (any dtype, head_dim <= 256, any block size / group)
// ---------------------------------------------------------------------------
constexpr int kSimtWarps = 4;
constexpr int kSimtMaxDPL = 8;  // dims per lane -> head_dim <= 256

struct SimtArgs {
  const void* q;
  int64_t q_sb, q_sh;
  OutTargets out;
  int64_t o_sb, o_sh;
  const void* k_pool;
  const void* v_pool;
  int64_t num_blocks, hkv, bs, d, layer;
  const int32_t* block_tables;
  int64_t bt_stride, bt_width;
  const int32_t* row_ids;
  const int32_t* seq_lens;
  int32_t g;
  float scale;
  int32_t* err;
};

template <typename T>
__global__ void __launch_bounds__(kSimtWarps * 32) decode_simt_kernel(const SimtArgs a) {
  __shared__ float s_o[kSimtWarps][kSimtMaxDPL * 32];
  __shared__ float s_m[kSimtWarps], s_l[kSimtWarps];
  const int b = blockIdx.x;
  const int hq = blockIdx.y;
  const int h = hq / a.g;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int len = a.seq_lens[b];
  const int64_t row = a.row_ids ? (int64_t)a.row_ids[b] : (int64_t)b;
  const T* qp = reinterpret_cast<const T*>(a.q) + (int64_t)b * a.q_sb + (int64_t)hq * a.q_sh;
  float qv[kSimtMaxDPL], ov[kSimtMaxDPL];
#pragma unroll
  for (int i = 0; i < kSimtMaxDPL; ++i) {
    const int d = lane + 32 * i;
    qv[i] = d < a.d ? to_f32<T>(qp[d]) : 0.f;
    ov[i] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  const T* kp = reinterpret_cast<const T*>(a.k_pool);
  const T* vp = reinterpret_cast<const T*>(a.v_pool);
  for (int t = warp; t < len; t += kSimtWarps) {
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
    for (int i = 0; i < kSimtMaxDPL; ++i) {
      const int d = lane + 32 * i;
      if (d < a.d) dot += qv[i] * to_f32<T>(kp[base + d]);
    }
#pragma unroll
    for (int off2 = 16; off2 > 0; off2 >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off2);
    const float s = dot * a.scale;
    const float mn = fmaxf(m, s);
    const float al = expf(m - mn);
    const float p = expf(s - mn);
    l = l * al + p;
#pragma unroll
    for (int i = 0; i < kSimtMaxDPL; ++i) {
      const int d = lane + 32 * i;
      ov[i] = ov[i] * al + (d < a.d ? p * to_f32<T>(vp[base + d]) : 0.f);
    }
    m = mn;
  }
#pragma unroll
  for (int i = 0; i < kSimtMaxDPL; ++i) s_o[warp][lane + 32 * i] = ov[i];
  if (lane == 0) {
    s_m[warp] = m;
    s_l[warp] = l;
  }
  __syncthreads();
  float M = -INFINITY;
  for (int w = 0; w < kSimtWarps; ++w) M = fmaxf(M, s_m[w]);
  const int64_t o_row = (int64_t)b * a.o_sb + (int64_t)hq * a.o_sh;
  for (int d = threadIdx.x; d < a.d; d += blockDim.x) {
    float L = 0.f, O = 0.f;
    for (int w = 0; w < kSimtWarps; ++w) {
      const float f = (s_m[w] == -INFINITY) ? 0.f : expf(s_m[w] - M);
      L += f * s_l[w];
      O += f * s_o[w][d];
    }
    store_targets<T>(a.out, o_row + d, from_f32<T>(L > 0.f ? O / L : 0.f));
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
bool tc_path(int32_t dtype, int64_t d, int64_t bs, int64_t hq, int64_t hkv) {
  if (dtype != BL_BF16 && dtype != BL_F16) return false;
  if (d != kD || bs != kBS) return false;
  if (hkv <= 0 || hq % hkv != 0) return false;
  const int64_t g = hq / hkv;
  return g >= 1 && g <= 8;
}

size_t tc_smem_bytes(int g) {
  return 1024 /*align slack*/ + kStages * kSlotBytes + (size_t)kNW * g * kD * sizeof(float) +
         kNW * 8 * 2 * sizeof(float) + sizeof(TCShared);
}

template <typename T>
int launch_tc_attention(const bl_decode_args& a, const OutTargets& ot, const WsLayout& w, cudaStream_t s) {
  const int g = (int)(a.num_q_heads / a.kv.num_kv_heads);
  const size_t smem = tc_smem_bytes(g);
  static int occ_cache[9] = {0};
  static std::mutex mu;
  int occ = 0;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (occ_cache[g] == 0) {
      if (cudaFuncSetAttribute(decode_tc_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)tc_smem_bytes(8)) != cudaSuccess) {
        set_error("decode: cudaFuncSetAttribute failed");
        return BL_ERR_LAUNCH;
      }
      int o = 0;
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, decode_tc_kernel<T>, kThreadsTC, smem);
      occ_cache[g] = o < 1 ? 1 : o;
    }
    occ = occ_cache[g];
  }

  const uint64_t rows = (uint64_t)a.kv.num_layers * a.kv.num_blocks * a.kv.num_kv_heads * kBS;
  CUtensorMap kmap, vmap;
  if (!get_pool_tmap(a.kv.k_pool, rows, a.kv.dtype, &kmap) ||
      !get_pool_tmap(a.kv.v_pool, rows, a.kv.dtype, &vmap))
    return BL_ERR_LAUNCH;

  char* ws = (char*)a.workspace;
  TCArgs k;
  k.q = a.q;
  k.q_sb = a.q_stride_b;
  k.q_sh = a.q_stride_h;
  k.out = ot;
  k.o_sb = a.out_stride_b;
  k.o_sh = a.out_stride_h;
  k.block_tables = a.kv.block_tables;
  k.bt_stride = a.kv.bt_stride;
  k.bt_width = (int32_t)std::min<int64_t>(a.kv.bt_width, INT32_MAX);
  k.row_ids = a.kv.row_ids;
  k.seq_lens = a.seq_lens;
  k.batch = (int32_t)a.batch;
  k.hq = (int32_t)a.num_q_heads;
  k.hkv = (int32_t)a.kv.num_kv_heads;
  k.g = g;
  k.num_blocks = a.kv.num_blocks;
  k.layer_row0 = (int64_t)a.kv.layer * a.kv.num_blocks * a.kv.num_kv_heads * kBS;
  k.scale_log2 = a.scale * kLog2e;
  k.chunk_blocks = kChunkTokens / kBS;
  k.hdr = (const int32_t*)(ws + w.hdr);
  k.row_base = (const int32_t*)(ws + w.row_base);
  k.exec = (const int2*)(ws + w.exec);
  k.ws_lse = (float*)(ws + w.lse);
  k.ws_o = (float*)(ws + w.o);
  k.max_units = (int32_t)w.max_units;
  k.err = a.err;

  const int64_t item_bound = w.max_units * a.kv.num_kv_heads;
  const int64_t grid = std::min<int64_t>((int64_t)num_sms() * occ, item_bound);
  if (launch_pdl(decode_tc_kernel<T>, dim3((unsigned)grid), dim3(kThreadsTC), smem, s, k, kmap, vmap) !=
      cudaSuccess) {
    set_error("decode_tc_kernel: launch failed: %s", cudaGetErrorString(cudaGetLastError()));
    return BL_ERR_LAUNCH;
  }
  return BL_OK;
}

template <typename T>
int launch_tc_reduce(const bl_decode_args& a, const OutTargets& ot, const WsLayout& w, cudaStream_t s) {
  char* ws = (char*)a.workspace;
  ReduceArgs r;
  r.out = ot;
  r.o_sb = a.out_stride_b;
  r.o_sh = a.out_stride_h;
  r.seq_lens = a.seq_lens;
  r.bs = kBS;
  r.chunk_blocks = kChunkTokens / kBS;
  r.bt_width = (int32_t)std::min<int64_t>(a.kv.bt_width, INT32_MAX);
  r.hq = (int32_t)a.num_q_heads;
  r.d = kD;
  r.row_base = (const int32_t*)(ws + w.row_base);
  r.ws_lse = (const float*)(ws + w.lse);
  r.ws_o = (const float*)(ws + w.o);
  r.max_units = (int32_t)w.max_units;
  if (launch_pdl(decode_reduce_kernel<T>, dim3((unsigned)a.batch, (unsigned)a.num_q_heads), dim3(kD), 0, s, r) !=
      cudaSuccess) {
    set_error("decode_reduce_kernel: launch failed: %s", cudaGetErrorString(cudaGetLastError()));
    return BL_ERR_LAUNCH;
  }
  return BL_OK;
}

template <typename T>
int launch_simt(const bl_decode_args& a, const OutTargets& ot, cudaStream_t s) {
  SimtArgs k;
  k.q = a.q;
  k.q_sb = a.q_stride_b;
  k.q_sh = a.q_stride_h;
  k.out = ot;
  k.o_sb = a.out_stride_b;
  k.o_sh = a.out_stride_h;
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
  k.seq_lens = a.seq_lens;
  k.g = (int32_t)(a.num_q_heads / a.kv.num_kv_heads);
  k.scale = a.scale;
  k.err = a.err;
  decode_simt_kernel<T><<<dim3((unsigned)a.batch, (unsigned)a.num_q_heads), kSimtWarps * 32, 0, s>>>(k);
  BL_CHECK_LAUNCH("decode_simt_kernel");
  return BL_OK;
}

int check_decode(const bl_decode_args* args, const char* who) {
  BL_CHECK_ARG(args != nullptr, "%s: args is null", who);
  const bl_decode_args& a = *args;
  int rc = check_paged_layer(a.kv, who);
  if (rc) return rc;
  BL_CHECK_ARG(a.q && a.out && a.seq_lens, "%s: null q/out/seq_lens", who);
  BL_CHECK_ARG(a.batch > 0 && a.batch <= 65535, "%s: batch must be in [1, 65535]", who);
  BL_CHECK_ARG(a.num_q_heads > 0 && a.num_q_heads <= 65535 &&
                   a.num_q_heads % a.kv.num_kv_heads == 0,
               "num_heads must divide evenly by num_kv_heads");
  BL_CHECK_ARG(a.kv.head_dim <= 256, "%s: head_dim > 256 is not supported", who);
  BL_CHECK_ARG(a.max_seq_len > 0, "KV cache is empty");
  return BL_OK;
}

}  // namespace
}  // namespace bl

using namespace bl;

extern "C" size_t bl_paged_decode_workspace_bytes(int64_t batch, int64_t num_q_heads, int64_t head_dim,
                                                  int64_t block_size, int64_t max_seq_len) {
  if (batch <= 0 || num_q_heads <= 0 || head_dim <= 0 || block_size <= 0 || max_seq_len <= 0) return 0;
  return ws_layout(batch, num_q_heads, head_dim, block_size, max_seq_len).total;
}

extern "C" int bl_decode_path(int32_t dtype, int64_t head_dim, int64_t block_size, int64_t num_q_heads,
                              int64_t num_kv_heads) {
  return tc_path(dtype, head_dim, block_size, num_q_heads, num_kv_heads) ? 1 : 0;
}

extern "C" int bl_paged_decode_plan(const bl_decode_args* args, void* stream) {
  int rc = check_decode(args, "bl_paged_decode_plan");
  if (rc) return rc;
  const bl_decode_args& a = *args;
  if (!tc_path(a.kv.dtype, a.kv.head_dim, a.kv.block_size, a.num_q_heads, a.kv.num_kv_heads))
    return BL_OK;  // the SIMT path needs no plan
  const WsLayout w = ws_layout(a.batch, a.num_q_heads, a.kv.head_dim, a.kv.block_size, a.max_seq_len);
  if (!a.workspace || a.workspace_bytes < w.total) {
    set_error("bl_paged_decode: workspace too small (%zu < %zu bytes)", a.workspace_bytes, w.total);
    return BL_ERR_CAPACITY;
  }
  BL_CHECK_ARG(((uintptr_t)a.workspace & 255) == 0, "bl_paged_decode: workspace must be 256-byte aligned");
  BL_CHECK_ARG(w.max_units <= INT32_MAX, "bl_paged_decode: too many split-K units");
  char* ws = (char*)a.workspace;
  PlanArgs p;
  p.seq_lens = a.seq_lens;
  p.batch = (int32_t)a.batch;
  p.bs = (int32_t)a.kv.block_size;
  p.chunk_blocks = kChunkTokens / kBS;
  p.bt_width = (int32_t)std::min<int64_t>(a.kv.bt_width, INT32_MAX);
  p.max_units = (int32_t)w.max_units;
  p.hdr = (int32_t*)(ws + w.hdr);
  p.row_base = (int32_t*)(ws + w.row_base);
  p.exec = (int2*)(ws + w.exec);
  p.err = a.err;
  if (launch_pdl(decode_plan_kernel, dim3(1), dim3(kPlanThreads), 0, (cudaStream_t)stream, p) != cudaSuccess) {
    set_error("decode_plan_kernel: launch failed: %s", cudaGetErrorString(cudaGetLastError()));
    return BL_ERR_LAUNCH;
  }
  return BL_OK;
}

namespace bl {
namespace {

// Validates the tensor-core-path specifics and the workspace; fills `w`.
int check_tc(const bl_decode_args& a, WsLayout& w) {
  const uint64_t rows = (uint64_t)a.kv.num_layers * a.kv.num_blocks * a.kv.num_kv_heads * kBS;
  BL_CHECK_ARG(rows <= (uint64_t)INT32_MAX, "bl_paged_decode: pool has more than 2^31 rows");
  BL_CHECK_ARG(((uintptr_t)a.kv.k_pool & 15) == 0 && ((uintptr_t)a.kv.v_pool & 15) == 0,
               "bl_paged_decode: pools must be 16-byte aligned");
  BL_CHECK_ARG(((uintptr_t)a.q & 3) == 0 && a.q_stride_b % 2 == 0 && a.q_stride_h % 2 == 0,
               "bl_paged_decode: q must be 4-byte aligned with even strides");
  w = ws_layout(a.batch, a.num_q_heads, a.kv.head_dim, a.kv.block_size, a.max_seq_len);
  if (!a.workspace || a.workspace_bytes < w.total) {
    set_error("bl_paged_decode: workspace too small (%zu < %zu bytes)", a.workspace_bytes, w.total);
    return BL_ERR_CAPACITY;
  }
  return BL_OK;
}

bool is_tc(const bl_decode_args& a) {
  return tc_path(a.kv.dtype, a.kv.head_dim, a.kv.block_size, a.num_q_heads, a.kv.num_kv_heads);
}

}  // namespace
}  // namespace bl

namespace bl {
namespace {

// The attention kernel of a checked call, storing to `targets`.
int decode_attention(const bl_decode_args& a, const OutTargets& targets, cudaStream_t s) {
  if (is_tc(a)) {
    WsLayout w;
    const int rc = check_tc(a, w);
    if (rc) return rc;
    OutTargets ot = targets;
    set_vec16(ot, a.out_stride_b, a.out_stride_h, elem_size(a.kv.dtype));
    if (a.kv.dtype == BL_BF16) return launch_tc_attention<__nv_bfloat16>(a, ot, w, s);
    return launch_tc_attention<__half>(a, ot, w, s);
  }
  const OutTargets& ot = targets;
  switch (a.kv.dtype) {
    case BL_F32: return launch_simt<float>(a, ot, s);
    case BL_F16: return launch_simt<__half>(a, ot, s);
    default: return launch_simt<__nv_bfloat16>(a, ot, s);
  }
}

// The split-K reduce of a checked call, storing to `targets`.
int decode_reduce(const bl_decode_args& a, const OutTargets& targets, cudaStream_t s) {
  if (!is_tc(a)) return BL_OK;  // the SIMT path never splits
  WsLayout w;
  const int rc = check_tc(a, w);
  if (rc) return rc;
  OutTargets ot = targets;
  set_vec16(ot, a.out_stride_b, a.out_stride_h, elem_size(a.kv.dtype));
  if (a.kv.dtype == BL_BF16) return launch_tc_reduce<__nv_bfloat16>(a, ot, w, s);
  return launch_tc_reduce<__half>(a, ot, w, s);
}

}  // namespace
}  // namespace bl

extern "C" int bl_paged_decode_attention(const bl_decode_args* args, void* stream) {
  const int rc = check_decode(args, "bl_paged_decode_attention");
  if (rc) return rc;
  return decode_attention(*args, one_target(args->out), (cudaStream_t)stream);
}

extern "C" int bl_paged_decode_reduce(const bl_decode_args* args, void* stream) {
  const int rc = check_decode(args, "bl_paged_decode_reduce");
  if (rc) return rc;
  return decode_reduce(*args, one_target(args->out), (cudaStream_t)stream);
}

extern "C" int bl_paged_decode(const bl_decode_args* args, void* stream) {
  int rc = check_decode(args, "bl_paged_decode");
  if (rc) return rc;
  if (is_tc(*args) && !args->plan_ready) {
    rc = bl_paged_decode_plan(args, stream);
    if (rc) return rc;
  }
  rc = bl_paged_decode_attention(args, stream);
  if (rc) return rc;
  return bl_paged_decode_reduce(args, stream);
}

// ---------------------------------------------------------------------------
// Allocation-free decode
// ---------------------------------------------------------------------------
// Some callers cannot hand this library a workspace: a host framework that
// owns every byte of device memory and passes plugins nothing but input and
// output pointers, or a latency-critical loop that must never enter
// cudaMalloc (which can synchronise the whole device).  For them,
// bl_paged_decode_noalloc runs the same split-K decode with its scratch in
// the fixed array below instead of a caller workspace.  The array is part of
// the library image: every GPU that loads the library keeps these 16 MiB for
// the life of the process.
namespace bl {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch on the current device.  In host code the
// symbol is only a stand-in, so the address is looked up once per device (the
// first call on that device does it, with that device current) and cached.
void* noalloc_scratch_on_current_device() {
  static std::mutex mu;
  static void* ptrs[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    set_error("bl_paged_decode_noalloc: cannot query the current device");
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_error("bl_paged_decode_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return nullptr;
    }
    ptrs[dev] = p;
  }
  return ptrs[dev];
}

}  // namespace
}  // namespace bl

extern "C" int bl_paged_decode_noalloc(const bl_decode_args* args, void* stream) {
  int rc = check_decode(args, "bl_paged_decode_noalloc");
  if (rc) return rc;
  bl_decode_args a = *args;
  if (is_tc(a)) {
    const WsLayout w = ws_layout(a.batch, a.num_q_heads, a.kv.head_dim, a.kv.block_size, a.max_seq_len);
    if (w.total > kNoAllocScratchBytes) {
      set_error("bl_paged_decode_noalloc: this batch needs %zu bytes of split-K scratch but the built-in scratch "
                "holds %zu; use bl_paged_decode with a caller workspace", w.total, kNoAllocScratchBytes);
      return BL_ERR_CAPACITY;
    }
    void* scratch = noalloc_scratch_on_current_device();
    if (!scratch) return BL_ERR_LAUNCH;
    a.workspace = scratch;
    a.workspace_bytes = kNoAllocScratchBytes;
  }
  // The plan is always rebuilt: the scratch holds whatever the previous call
  // left there.  Nothing in it has to start at zero -- the plan kernel writes
  // every entry the attention and reduce kernels read.
  a.plan_ready = 0;
  return bl_paged_decode(&a, stream);
}

// ---------------------------------------------------------------------------
// KV-head-sharded decode with the output all-gather fused into the epilogue
// ---------------------------------------------------------------------------
// Each rank runs the ordinary plan / attention / reduce over its own heads;
// the only difference is the output: every element goes to all ranks'
// gathered buffers at this rank's head offset (rank r + j first, so the
// ranks do not all write to the same peer at once), and a barrier kernel
// closes the call.
extern "C" int bl_paged_decode_allgather(const bl_decode_args* args, const bl_head_gather* gather, void* stream) {
  const char* who = "bl_paged_decode_allgather";
  BL_CHECK_ARG(args != nullptr && gather != nullptr, "%s: null argument", who);
  int rc = check_head_gather(*gather, who);
  if (rc) return rc;
  const bl_head_gather& g = *gather;
  bl_decode_args a = *args;
  const int es = elem_size(a.kv.dtype);
  BL_CHECK_ARG(es > 0, "%s: unsupported dtype code %d", who, a.kv.dtype);
  const int64_t head_bytes = g.head_offset * a.out_stride_h * es;
  a.out = (char*)g.peer_out[g.rank] + head_bytes;
  rc = check_decode(&a, who);
  if (rc) return rc;
  OutTargets ot = {};
  ot.n = g.world;
  for (int j = 0; j < g.world; ++j) ot.ptr[j] = (char*)g.peer_out[(g.rank + j) % g.world] + head_bytes;
  cudaStream_t s = (cudaStream_t)stream;
  if (is_tc(a) && !a.plan_ready) {
    rc = bl_paged_decode_plan(&a, stream);
    if (rc) return rc;
  }
  rc = decode_attention(a, ot, s);
  if (rc) return rc;
  rc = decode_reduce(a, ot, s);
  if (rc) return rc;
  return launch_peer_barrier(g, a.err, s);
}
