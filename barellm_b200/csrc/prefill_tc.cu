// Tensor-core paged chunked-prefill attention (bf16 / fp16, head_dim 128,
// block_size 16, GQA group G in {1, 2, 4, 8}).
//
// One CTA owns a tile of 128 score rows = (128 / G) query tokens x the G
// query heads sharing one KV head, so each K/V page is loaded once for the
// whole GQA group.  Rows are head-major: warp w holds rows 16w..16w+15, i.e.
// 16 consecutive query tokens of one query head.
//   producer warp : one lane streams the row's pages through the block table,
//                   4 pages (64 keys, 32 KiB of K+V) per stage, 3 stages, with
//                   2-D TMA and the 128-byte swizzle.
//   8 consumer warps : S = Q K^T and O += P V on mma.sync m16n8k16 with fp32
//                   accumulators; Q stays in registers; online softmax in fp32;
//                   the bottom-right causal mask is applied only on the tiles
//                   that straddle a warp's diagonal.
// Roofline: tensor.  Algorithmic flops per row = 4 * Hq * D * (C*P + C(C+1)/2).
#include "prefill_tc.cuh"

namespace bl {
namespace {

constexpr int kD = 128;
constexpr int kBS = 16;
constexpr int kPPT = 4;                       // pages per key tile
constexpr int kKT = kPPT * kBS;               // 64 keys per tile
constexpr int kNW = 8;                        // consumer warps
constexpr int kThreads = (kNW + 1) * 32;
constexpr int kStages = 3;
constexpr int kPage = kBS * kD * 2;           // 4 KiB
constexpr int kStageBytes = kPPT * 2 * kPage; // 32 KiB
constexpr int kRows = kNW * 16;               // 128 score rows per CTA
constexpr float kLog2e = 1.4426950408889634f;

struct PArgs {
  const void* q;
  int64_t q_sb, q_st, q_sh;
  void* out;
  int64_t o_sb, o_st, o_sh;
  const int32_t* q_offsets;
  const int32_t* seq_lens;
  const int32_t* block_tables;
  int64_t bt_stride;
  int32_t bt_width;
  const int32_t* row_ids;
  int32_t hkv, g, bq;
  int64_t num_blocks, layer_row0, max_q;
  float scale_log2;
  int32_t* err;
};

struct PShared {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  int abort;
};

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_tc_kernel(const PArgs a, const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  PShared* sh = reinterpret_cast<PShared*>(smem + kStages * kStageBytes);

  // heaviest tiles (latest queries, most keys) are launched first
  const int64_t qtile = (int64_t)gridDim.x - 1 - blockIdx.x;
  const int h = blockIdx.y;
  const int64_t b = blockIdx.z;
  int64_t qo = 0, nq = a.max_q;
  if (a.q_offsets) {
    qo = a.q_offsets[b];
    nq = (int64_t)a.q_offsets[b + 1] - qo;
  }
  const int64_t q0 = qtile * a.bq;
  if (q0 >= nq) return;
  const int64_t len = a.seq_lens[b];
  const int64_t prefix = len - nq;
  const int64_t kend = prefix + min(q0 + (int64_t)a.bq, nq);  // keys [0, kend)
  int npages = (int)((kend + kBS - 1) / kBS);
  if (npages > a.bt_width) npages = a.bt_width;  // reported by the producer
  const int ntiles = (npages + kPPT - 1) / kPPT;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sh->full[s], 1);
      mbar_init(&sh->empty[s], kNW);
    }
    sh->abort = 0;
    fence_mbar_init();
  }
  __syncthreads();

  const int64_t row = a.row_ids ? (int64_t)a.row_ids[b] : b;
  if (warp == kNW) {
    // ------------------------------ producer ------------------------------
    if (lane != 0) return;
    if ((int)((kend + kBS - 1) / kBS) > a.bt_width) raise_dev(a.err, BL_DEVERR_TABLE);
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
    const int32_t* bt = a.block_tables + row * a.bt_stride;
    int issued = 0;
    for (int t = 0; t < ntiles; ++t) {
      const int slot = t % kStages;
      if (!mbar_wait(&sh->empty[slot], ((t / kStages) & 1) ^ 1)) {
        raise_dev(a.err, BL_DEVERR_TIMEOUT);
        sh->abort = 1;
        break;
      }
      const int np = min(kPPT, npages - t * kPPT);
      unsigned char* st = smem + slot * kStageBytes;
      mbar_arrive_expect_tx(&sh->full[slot], np * 2 * kPage);
      for (int p = 0; p < np; ++p) {
        int64_t phys = bt[t * kPPT + p];
        if (phys < 0 || phys >= a.num_blocks) {
          raise_dev(a.err, BL_DEVERR_BLOCK_ID);
          phys = 0;
        }
        const int32_t y = (int32_t)(a.layer_row0 + (phys * a.hkv + h) * kBS);
        unsigned char* kd = st + p * kPage;
        unsigned char* vd = st + kPPT * kPage + p * kPage;
        tma_load_2d(kd, &kmap, &sh->full[slot], 0, y);
        tma_load_2d(kd + kPage / 2, &kmap, &sh->full[slot], 64, y);
        tma_load_2d(vd, &vmap, &sh->full[slot], 0, y);
        tma_load_2d(vd + kPage / 2, &vmap, &sh->full[slot], 64, y);
      }
      ++issued;
    }
    for (int s = 0; s < kStages && s < issued; ++s) {
      const int last = s + ((issued - 1 - s) / kStages) * kStages;
      if (!mbar_wait(&sh->full[s], (last / kStages) & 1)) raise_dev(a.err, BL_DEVERR_TIMEOUT);
    }
    return;
  }

  // ------------------------------ consumers ------------------------------
  const int g_row = lane >> 2;
  const int t4 = lane & 3;
  const int m0 = warp * 16;
  const int hd = m0 / a.bq;
  const int tok0 = m0 - hd * a.bq;
  const int hq = h * a.g + hd;
  const int64_t i0 = q0 + tok0 + g_row;  // query index of rows g_row / g_row + 8
  const int64_t i1 = i0 + 8;
  const bool v0 = i0 < nq, v1 = i1 < nq;
  const int64_t lim0 = prefix + i0, lim1 = prefix + i1;  // inclusive key limits
  const int64_t warp_min_lim = prefix + q0 + tok0;
  const int64_t warp_max_lim = prefix + min(q0 + tok0 + 15, nq - 1);

  uint32_t qf[8][4];
  {
    const T* qb = reinterpret_cast<const T*>(a.q) + b * a.q_sb + (int64_t)hq * a.q_sh;
    const T* q0p = qb + (qo + (v0 ? i0 : 0)) * a.q_st;
    const T* q1p = qb + (qo + (v1 ? i1 : 0)) * a.q_st;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const int c = ks * 16 + 2 * t4;
      qf[ks][0] = v0 ? *reinterpret_cast<const uint32_t*>(q0p + c) : 0u;
      qf[ks][1] = v1 ? *reinterpret_cast<const uint32_t*>(q1p + c) : 0u;
      qf[ks][2] = v0 ? *reinterpret_cast<const uint32_t*>(q0p + c + 8) : 0u;
      qf[ks][3] = v1 ? *reinterpret_cast<const uint32_t*>(q1p + c + 8) : 0u;
    }
  }

  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float mr0 = -INFINITY, mr1 = -INFINITY, lr0 = 0.f, lr1 = 0.f;

  // per-lane ldmatrix geometry
  const int key_k = (lane & 7) + ((lane >> 4) << 3);  // K (non-trans) rows
  const int hi_k = (lane >> 3) & 1;
  const int key_v = (lane & 7) + (((lane >> 3) & 1) << 3);  // V (trans) rows
  const int hi_v = lane >> 4;

  for (int t = 0; t < ntiles; ++t) {
    const int slot = t % kStages;
    if (*(volatile int*)&sh->abort) break;
    if (!mbar_wait(&sh->full[slot], (t / kStages) & 1)) {
      raise_dev(a.err, BL_DEVERR_TIMEOUT);
      *(volatile int*)&sh->abort = 1;
      break;
    }
    const int np = min(kPPT, npages - t * kPPT);
    const int64_t kt0 = (int64_t)t * kKT;
    if (kt0 <= warp_max_lim) {
      const uint32_t kst = smem_u32(smem + slot * kStageBytes);
      const uint32_t vst = kst + kPPT * kPage;
      float s[8][4];
#pragma unroll
      for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const int cc = 2 * (ks & 3) + hi_k;
        const uint32_t off = (ks >> 2) * (kPage / 2) + key_k * 128 + ((cc ^ (key_k & 7)) << 4);
#pragma unroll
        for (int p = 0; p < kPPT; ++p) {
          if (p < np) {
            uint32_t r0, r1, r2, r3;
            ldmatrix_x4(kst + p * kPage + off, r0, r1, r2, r3);
            mma_16816<T>(s[2 * p][0], s[2 * p][1], s[2 * p][2], s[2 * p][3], qf[ks][0], qf[ks][1],
                         qf[ks][2], qf[ks][3], r0, r1);
            mma_16816<T>(s[2 * p + 1][0], s[2 * p + 1][1], s[2 * p + 1][2], s[2 * p + 1][3],
                         qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3], r2, r3);
          }
        }
      }
      // scale + causal mask (only where this tile crosses the warp's diagonal)
      const bool need_mask = (kt0 + kKT - 1 > warp_min_lim) || (np < kPPT);
#pragma unroll
      for (int n = 0; n < 8; ++n) {
#pragma unroll
        for (int c = 0; c < 4; ++c) s[n][c] *= a.scale_log2;
        if (need_mask) {
          const int64_t key = kt0 + 8 * n + 2 * t4;
          const bool loaded = (n >> 1) < np;
          if (!loaded || key > lim0) s[n][0] = -INFINITY;
          if (!loaded || key + 1 > lim0) s[n][1] = -INFINITY;
          if (!loaded || key > lim1) s[n][2] = -INFINITY;
          if (!loaded || key + 1 > lim1) s[n][3] = -INFINITY;
        }
      }
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        mx0 = fmaxf(mx0, fmaxf(s[n][0], s[n][1]));
        mx1 = fmaxf(mx1, fmaxf(s[n][2], s[n][3]));
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float mn0 = fmaxf(mr0, mx0), mn1 = fmaxf(mr1, mx1);
      const float ms0 = (mn0 == -INFINITY) ? 0.f : mn0;  // fully masked so far
      const float ms1 = (mn1 == -INFINITY) ? 0.f : mn1;
      const float al0 = fast_exp2(mr0 - ms0), al1 = fast_exp2(mr1 - ms1);
      mr0 = mn0;
      mr1 = mn1;
      float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        s[n][0] = fast_exp2(s[n][0] - ms0);
        s[n][1] = fast_exp2(s[n][1] - ms0);
        s[n][2] = fast_exp2(s[n][2] - ms1);
        s[n][3] = fast_exp2(s[n][3] - ms1);
        rs0 += s[n][0] + s[n][1];
        rs1 += s[n][2] + s[n][3];
      }
      lr0 = lr0 * al0 + rs0;
      lr1 = lr1 * al1 + rs1;
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        o[n][0] *= al0;
        o[n][1] *= al0;
        o[n][2] *= al1;
        o[n][3] *= al1;
      }
      // O += P V
#pragma unroll
      for (int kk = 0; kk < kPPT; ++kk) {
        if (kk < np) {
          const uint32_t pa0 = pack2<T>(s[2 * kk][0], s[2 * kk][1]);
          const uint32_t pa1 = pack2<T>(s[2 * kk][2], s[2 * kk][3]);
          const uint32_t pa2 = pack2<T>(s[2 * kk + 1][0], s[2 * kk + 1][1]);
          const uint32_t pa3 = pack2<T>(s[2 * kk + 1][2], s[2 * kk + 1][3]);
          // keys past the row length hold stale pool bytes: zero them
          const int64_t pk0 = kt0 + kk * kBS;
          uint32_t mlo = 0xffffffffu, mhi = 0xffffffffu;
          if (pk0 + kBS > len) {
            const int64_t nv = len - pk0;
            mlo = (2 * t4 < nv ? 0x0000ffffu : 0u) | (2 * t4 + 1 < nv ? 0xffff0000u : 0u);
            mhi = (8 + 2 * t4 < nv ? 0x0000ffffu : 0u) | (9 + 2 * t4 < nv ? 0xffff0000u : 0u);
          }
          const uint32_t vpg = vst + kk * kPage;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int cc = 2 * (j & 3) + hi_v;
            const uint32_t addr = vpg + (j >> 2) * (kPage / 2) + key_v * 128 + ((cc ^ (key_v & 7)) << 4);
            uint32_t r0, r1, r2, r3;
            ldmatrix_x4_trans(addr, r0, r1, r2, r3);
            mma_16816<T>(o[2 * j][0], o[2 * j][1], o[2 * j][2], o[2 * j][3], pa0, pa1, pa2, pa3,
                         r0 & mlo, r1 & mhi);
            mma_16816<T>(o[2 * j + 1][0], o[2 * j + 1][1], o[2 * j + 1][2], o[2 * j + 1][3], pa0, pa1,
                         pa2, pa3, r2 & mlo, r3 & mhi);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sh->empty[slot]);
  }

  // ---- epilogue: normalise and store ----
  lr0 += __shfl_xor_sync(0xffffffffu, lr0, 1);
  lr0 += __shfl_xor_sync(0xffffffffu, lr0, 2);
  lr1 += __shfl_xor_sync(0xffffffffu, lr1, 1);
  lr1 += __shfl_xor_sync(0xffffffffu, lr1, 2);
  const float inv0 = lr0 > 0.f ? 1.f / lr0 : 0.f;
  const float inv1 = lr1 > 0.f ? 1.f / lr1 : 0.f;
  T* ob = reinterpret_cast<T*>(a.out) + b * a.o_sb + (int64_t)hq * a.o_sh;
  if (v0) {
    T* op = ob + (qo + i0) * a.o_st;
#pragma unroll
    for (int n = 0; n < 16; ++n)
      *reinterpret_cast<uint32_t*>(op + 8 * n + 2 * t4) = pack2<T>(o[n][0] * inv0, o[n][1] * inv0);
  }
  if (v1) {
    T* op = ob + (qo + i1) * a.o_st;
#pragma unroll
    for (int n = 0; n < 16; ++n)
      *reinterpret_cast<uint32_t*>(op + 8 * n + 2 * t4) = pack2<T>(o[n][2] * inv1, o[n][3] * inv1);
  }
}

size_t smem_bytes() { return 1024 + kStages * kStageBytes + sizeof(PShared); }

template <typename T>
int launch(const bl_prefill_args& a, cudaStream_t s) {
  static bool attr_done = false;
  if (!attr_done) {
    if (cudaFuncSetAttribute(prefill_tc_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem_bytes()) != cudaSuccess) {
      set_error("prefill: cudaFuncSetAttribute failed");
      return BL_ERR_LAUNCH;
    }
    attr_done = true;
  }
  const uint64_t rows = (uint64_t)a.kv.num_layers * a.kv.num_blocks * a.kv.num_kv_heads * kBS;
  CUtensorMap kmap, vmap;
  if (!get_pool_tmap(a.kv.k_pool, rows, a.kv.dtype, &kmap) ||
      !get_pool_tmap(a.kv.v_pool, rows, a.kv.dtype, &vmap))
    return BL_ERR_LAUNCH;
  PArgs k;
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
  k.block_tables = a.kv.block_tables;
  k.bt_stride = a.kv.bt_stride;
  k.bt_width = (int32_t)std::min<int64_t>(a.kv.bt_width, INT32_MAX);
  k.row_ids = a.kv.row_ids;
  k.hkv = (int32_t)a.kv.num_kv_heads;
  k.g = (int32_t)(a.num_q_heads / a.kv.num_kv_heads);
  k.bq = kRows / k.g;
  k.num_blocks = a.kv.num_blocks;
  k.layer_row0 = (int64_t)a.kv.layer * a.kv.num_blocks * a.kv.num_kv_heads * kBS;
  k.max_q = a.max_q_len;
  k.scale_log2 = a.scale * kLog2e;
  k.err = a.err;
  const int64_t tiles = (a.max_q_len + k.bq - 1) / k.bq;
  dim3 grid((unsigned)tiles, (unsigned)a.kv.num_kv_heads, (unsigned)a.batch);
  prefill_tc_kernel<T><<<grid, kThreads, smem_bytes(), s>>>(k, kmap, vmap);
  BL_CHECK_LAUNCH("prefill_tc_kernel");
  return BL_OK;
}

}  // namespace

bool prefill_tc_supported(int32_t dtype, int64_t head_dim, int64_t block_size, int64_t hq, int64_t hkv) {
  if (dtype != BL_BF16 && dtype != BL_F16) return false;
  if (head_dim != kD || block_size != kBS) return false;
  if (hkv <= 0 || hq % hkv != 0) return false;
  const int64_t g = hq / hkv;
  return g == 1 || g == 2 || g == 4 || g == 8;
}

int prefill_tc_launch(const bl_prefill_args& a, cudaStream_t s) {
  const uint64_t rows = (uint64_t)a.kv.num_layers * a.kv.num_blocks * a.kv.num_kv_heads * kBS;
  BL_CHECK_ARG(rows <= (uint64_t)INT32_MAX, "bl_paged_prefill: pool has more than 2^31 rows");
  BL_CHECK_ARG(((uintptr_t)a.kv.k_pool & 15) == 0 && ((uintptr_t)a.kv.v_pool & 15) == 0,
               "bl_paged_prefill: pools must be 16-byte aligned");
  BL_CHECK_ARG(((uintptr_t)a.q & 3) == 0 && ((uintptr_t)a.out & 3) == 0 && a.q_stride_b % 2 == 0 &&
                   a.q_stride_t % 2 == 0 && a.q_stride_h % 2 == 0 && a.out_stride_b % 2 == 0 &&
                   a.out_stride_t % 2 == 0 && a.out_stride_h % 2 == 0,
               "bl_paged_prefill: q/out must be 4-byte aligned with even strides");
  if (a.kv.dtype == BL_BF16) return launch<__nv_bfloat16>(a, s);
  return launch<__half>(a, s);
}

}  // namespace bl
