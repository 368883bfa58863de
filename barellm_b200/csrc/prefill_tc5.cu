// Paged chunked-prefill attention on 5th-generation tensor cores (tcgen05 +
// tensor memory), bf16 / fp16, head_dim 128, block_size 16, GQA group G in
// {1, 2, 4, 8}.
//
// A CTA owns 128 score rows = (128 / G) query tokens x the G query heads that
// share one KV head (head-major: row r = head (r / bq), token (r % bq)), so
// every K/V page is fetched once for the whole GQA group.  Keys are consumed
// in tiles of 128 (8 pages).  Warp roles:
//   warp 0      TMA producer: K and V pages of a tile, each page two 64 x 16
//               boxes with the 128-byte swizzle, into a 2-stage ring with
//               separate K and V slots.  K runs a tile ahead of V: a K slot is
//               recycled as soon as its S = Q K^T MMAs finish, a V slot only
//               after its P V MMAs.  Pages past the row's last page are fetched
//               from out-of-range coordinates, which TMA fills with zeros.
//   warp 1      TMEM owner (512 columns: S double buffer at 0 / 128, O at 256)
//               and, on one lane, the MMA issuer: S_t = Q K_t^T (M 128, N 128,
//               8 x K16, both operands K-major) into S[t % 2], then
//               O += P_{t-1} V_{t-1} (P K-major from shared memory, V MN-major).
//   warps 2..9  softmax + epilogue, two threads per score row (= TMEM lane),
//               each owning 64 of its columns; per tile they exchange only the
//               row max.  tcgen05.ld the S half-row, scale to log2 units,
//               bottom-right causal mask, online softmax with a lazy rescale (O
//               in TMEM is rescaled only when the running max grows by more
//               than 2^8), exponentials computed while the previous P V still
//               runs, P as bf16/fp16 into the swizzled shared P tile; finally
//               O / l from TMEM to global memory.
// Every mbarrier wait is bounded; on a time-out the CTA records
// BL_DEVERR_TIMEOUT, drains what it issued and frees its TMEM.
// Roofline: tensor.  Algorithmic flops per request: 4 * Hq * D * (C*P + C(C+1)/2).
#include <type_traits>

#include "prefill_tc.cuh"

namespace bl {
namespace {

constexpr int kD = 128;
constexpr int kBS = 16;
constexpr int kKT = 128;                 // keys per tile
constexpr int kPPT = kKT / kBS;          // 8 pages per tile
constexpr int kRows = 128;               // score rows per CTA (MMA M)
constexpr int kStages = 2;
constexpr int kThreads = 320;            // producer, MMA, 8 softmax warps
constexpr int kSoftmaxThreads = 256;
constexpr int kHalf = 128 * 128;         // 16 KB: 128 rows x 128 B (64 elements of D or K)
constexpr int kTile = 2 * kHalf;         // 32 KB
constexpr int kPageHalf = kBS * 128;     // 2 KB: 16 rows x 128 B
constexpr int kOffQ = 0;
constexpr int kOffK = kTile;                    // + s * kTile
constexpr int kOffV = kOffK + kStages * kTile;  // + s * kTile
constexpr int kOffP = kOffV + kStages * kTile;
constexpr int kSmemData = kOffP + kTile;        // 192 KB
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0;                   // + buffer * 128
constexpr uint32_t kColO = 256;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;       // log2 units

struct Args {
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
  int32_t rows_total;  // rows of the pool tensor map: an out-of-range coordinate
  float scale_log2;
  int32_t* err;
};

struct Shared {
  uint64_t full_k[kStages], full_v[kStages], empty_k[kStages], empty_v[kStages];
  uint64_t s_full[2], s_free[2], p_full, pv_done, q_full, mma_done;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, Shared* sh, int32_t* err) {
  if (*(volatile int*)&sh->abort) return false;
  if (mbar_wait(bar, parity)) return true;
  raise_dev(err, BL_DEVERR_TIMEOUT);
  *(volatile int*)&sh->abort = 1;
  return false;
}

template <bool BF16>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_tc5_kernel(const Args a, const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap) {
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Shared* sh = reinterpret_cast<Shared*>(smem + kSmemData);

  // ---- which 128 rows: heaviest q tiles first ----
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
  const bool table_short = npages > a.bt_width;
  if (table_short) npages = a.bt_width;
  const int ntiles = (npages + kPPT - 1) / kPPT;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sh->full_k[s], 1);
      mbar_init(&sh->full_v[s], 1);
      mbar_init(&sh->empty_k[s], 1);
      mbar_init(&sh->empty_v[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sh->s_full[i], 1);
      mbar_init(&sh->s_free[i], kSoftmaxThreads);
    }
    mbar_init(&sh->p_full, kSoftmaxThreads);
    mbar_init(&sh->pv_done, 1);
    mbar_init(&sh->q_full, kSoftmaxThreads);
    mbar_init(&sh->mma_done, 1);
    sh->abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) tc_alloc(&sh->tmem_base, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;

  if (warp == 0) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      if (table_short) raise_dev(a.err, BL_DEVERR_TABLE);
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
      const int64_t row = a.row_ids ? (int64_t)a.row_ids[b] : b;
      const int32_t* bt = a.block_tables + row * a.bt_stride;
      int issued_k = 0, issued_v = 0;
      auto page_rows = [&](int t, int32_t(&ys)[kPPT]) {
        for (int p = 0; p < kPPT; ++p) {
          const int lb = t * kPPT + p;
          if (lb < npages) {
            int64_t phys = bt[lb];
            if (phys < 0 || phys >= a.num_blocks) {
              raise_dev(a.err, BL_DEVERR_BLOCK_ID);
              phys = 0;
            }
            ys[p] = (int32_t)(a.layer_row0 + (phys * a.hkv + h) * kBS);
          } else {
            ys[p] = a.rows_total;  // fully out of range: TMA writes zeros
          }
        }
      };
      auto load = [&](const CUtensorMap* map, uint64_t* full, unsigned char* dst, int t) {
        int32_t ys[kPPT];
        page_rows(t, ys);
        mbar_arrive_expect_tx(full, kTile);
        for (int p = 0; p < kPPT; ++p) {
          tma_load_2d(dst + p * kPageHalf, map, full, 0, ys[p]);
          tma_load_2d(dst + kHalf + p * kPageHalf, map, full, 64, ys[p]);
        }
      };
      // K runs one tile ahead of V: K slots free up right after S = Q K^T,
      // V slots only after P V, so waiting on a V slot must not hold back K.
      for (int t = 0; t <= ntiles; ++t) {
        if (t < ntiles) {
          const int s = t & 1;
          if (!wait_or_abort(&sh->empty_k[s], ((t >> 1) & 1) ^ 1, sh, a.err)) break;
          load(&kmap, &sh->full_k[s], smem + kOffK + s * kTile, t);
          ++issued_k;
        }
        if (t >= 1) {
          const int j = t - 1, s = j & 1;
          if (!wait_or_abort(&sh->empty_v[s], ((j >> 1) & 1) ^ 1, sh, a.err)) break;
          load(&vmap, &sh->full_v[s], smem + kOffV + s * kTile, j);
          ++issued_v;
        }
      }
      // drain: every issued copy must land before the CTA can exit
      for (int s = 0; s < kStages; ++s) {
        if (s < issued_k) {
          const int last = s + ((issued_k - 1 - s) / kStages) * kStages;
          if (!mbar_wait(&sh->full_k[s], (last >> 1) & 1)) raise_dev(a.err, BL_DEVERR_TIMEOUT);
        }
        if (s < issued_v) {
          const int last = s + ((issued_v - 1 - s) / kStages) * kStages;
          if (!mbar_wait(&sh->full_v[s], (last >> 1) & 1)) raise_dev(a.err, BL_DEVERR_TIMEOUT);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ------------------------------
    if (lane == 0) {
      const uint32_t idesc_s = umma_idesc_f16(kRows, kKT, BF16, false);
      const uint32_t idesc_o = umma_idesc_f16(kRows, kD, BF16, true);
      const uint32_t sq = smem_u32(smem + kOffQ);
      const uint32_t sp = smem_u32(smem + kOffP);
      bool ok = wait_or_abort(&sh->q_full, 0, sh, a.err);
      auto issue_pv = [&](int j) -> bool {
        const int s = j & 1;
        if (!wait_or_abort(&sh->full_v[s], (j >> 1) & 1, sh, a.err)) return false;
        if (!wait_or_abort(&sh->p_full, j & 1, sh, a.err)) return false;
        tc_fence_after();
        const uint32_t sv = smem_u32(smem + kOffV + s * kTile);
#pragma unroll
        for (int kk = 0; kk < kKT / 16; ++kk) {
          const uint64_t da = umma_desc_sw128(sp + (kk >> 2) * kHalf + (kk & 3) * 32, 16, 1024);
          const uint64_t db = umma_desc_sw128(sv + kk * 2048, kHalf, 1024);
          tc_mma_ss(tmem + kColO, da, db, idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(&sh->pv_done);
        tc_commit(&sh->empty_v[s]);
        return true;
      };
      if (ok) tc_fence_after();
      for (int t = 0; t < ntiles && ok; ++t) {
        const int s = t & 1;
        ok = wait_or_abort(&sh->full_k[s], (t >> 1) & 1, sh, a.err) &&
             wait_or_abort(&sh->s_free[s], ((t >> 1) & 1) ^ 1, sh, a.err);
        if (!ok) break;
        tc_fence_after();
        const uint32_t sk = smem_u32(smem + kOffK + s * kTile);
#pragma unroll
        for (int ks = 0; ks < kD / 16; ++ks) {
          const uint32_t off = (ks >> 2) * kHalf + (ks & 3) * 32;
          tc_mma_ss(tmem + kColS + s * kKT, umma_desc_sw128(sq + off, 16, 1024), umma_desc_sw128(sk + off, 16, 1024),
                    idesc_s, ks > 0 ? 1u : 0u);
        }
        tc_commit(&sh->s_full[s]);
        tc_commit(&sh->empty_k[s]);
        if (t >= 1) ok = issue_pv(t - 1);
      }
      if (ok && ntiles > 0) ok = issue_pv(ntiles - 1);
      // every MMA issued here has finished before the CTA tears down
      tc_commit(&sh->mma_done);
      if (!mbar_wait(&sh->mma_done, 0)) raise_dev(a.err, BL_DEVERR_TIMEOUT);
    }
  } else {
    // ------------------------------ softmax ------------------------------
    // Two threads per score row: warps w and w+4 share the TMEM lane group
    // (w % 4) and split the row's 128 columns (keys of S / dims of O) in two
    // halves; only the row max is exchanged per tile.
    const int sw = warp - 2;                // 0..7
    const int half = sw >> 2;               // 0: columns 0-63, 1: columns 64-127
    const int grp = warp & 3;               // TMEM lane group
    const int r = 32 * grp + lane;          // score row == TMEM lane
    const uint32_t tl = tmem + ((uint32_t)(32 * grp) << 16) + half * 64;
    float* red = reinterpret_cast<float*>(sh + 1);          // [2][kRows] partial maxima / sums
    int* red_ok = reinterpret_cast<int*>(red + 2 * kRows);  // [2][kRows]
    const int pair_bar = 2 + grp;           // named barrier shared by the two warps of a row group
    const int hd = r / a.bq;
    const int tok = r - hd * a.bq;
    const int64_t qi = q0 + tok;
    const bool valid = qi < nq;
    const int hq = h * a.g + hd;
    const int64_t lim = prefix + qi;  // inclusive key limit
    // this thread's half of the Q row -> shared memory (K-major, 128-byte swizzle)
    {
      const T* qrow = reinterpret_cast<const T*>(a.q) + b * a.q_sb + (qo + (valid ? qi : 0)) * a.q_st +
                      (int64_t)hq * a.q_sh + half * 64;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint4 v = make_uint4(0, 0, 0, 0);
        if (valid) {
          const uint32_t* src = reinterpret_cast<const uint32_t*>(qrow + c * 8);
          v = make_uint4(src[0], src[1], src[2], src[3]);
        }
        *reinterpret_cast<uint4*>(smem + kOffQ + half * kHalf + r * 128 + ((c ^ (r & 7)) << 4)) = v;
      }
    }
    fence_proxy_async_smem();
    mbar_arrive(&sh->q_full);

    // A failed (timed-out) wait never makes one warp of a pair leave the loop
    // early: both always reach the pair barriers, agree on the failure there,
    // and skip the remaining work together.
    float m_used = -INFINITY, l = 0.f;
    bool failed = false;
    for (int t = 0; t < ntiles; ++t) {
      const int s = t & 1;
      bool ok = !failed && __all_sync(0xffffffffu, wait_or_abort(&sh->s_full[s], (t >> 1) & 1, sh, a.err));
      float x[64];
      float mt = -INFINITY;
      const int64_t k0 = (int64_t)t * kKT + half * 64;
      if (ok) {
        tc_fence_after();
        tc_ld32f(tl + kColS + s * kKT, x);
        tc_ld32f(tl + kColS + s * kKT + 32, x + 32);
        tc_wait_ld();
#pragma unroll
        for (int j = 0; j < 64; ++j) x[j] *= a.scale_log2;
        tc_fence_before();
        mbar_arrive(&sh->s_free[s]);
        if (k0 + 63 > lim) {
#pragma unroll
          for (int j = 0; j < 64; ++j)
            if (k0 + j > lim) x[j] = -INFINITY;
        }
#pragma unroll
        for (int j = 0; j < 64; ++j) mt = fmaxf(mt, x[j]);
      }
      red[half * kRows + r] = mt;
      red_ok[half * kRows + r] = ok ? 1 : 0;
      named_barrier_sync(pair_bar, 64);
      mt = fmaxf(mt, red[(half ^ 1) * kRows + r]);
      ok = ok && red_ok[(half ^ 1) * kRows + r] != 0;
      named_barrier_sync(pair_bar, 64);  // the slots are rewritten next tile
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        failed = true;
        continue;
      }
      const float m_new = fmaxf(m_used, mt);
      const bool need = (t > 0) && (m_new > m_used + kRescaleThreshold);
      // the exponentials need only the new max, so they overlap the previous
      // tile's P V; O and the P buffer are touched only after it completes
      const float alpha = need ? fast_exp2(m_used - m_new) : 1.f;
      if (need || t == 0) m_used = m_new;
      const float ms = (m_used == -INFINITY) ? 0.f : m_used;
      float rs = 0.f;
#pragma unroll
      for (int j = 0; j < 64; ++j) {
        x[j] = fast_exp2(x[j] - ms);
        rs += x[j];
      }
      l = l * alpha + rs;
      if (t >= 1) {
        if (!__all_sync(0xffffffffu, wait_or_abort(&sh->pv_done, (t - 1) & 1, sh, a.err))) {
          failed = true;
          continue;
        }
        tc_fence_after();
      }
      // P (keys of this half) into the half of the swizzled P tile it owns;
      // packing first frees the fp32 row before O is rescaled
      unsigned char* prow = smem + kOffP + half * kHalf + r * 128;
      uint32_t pk[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) pk[e] = pack2<T>(x[2 * e], x[2 * e + 1]);
#pragma unroll
      for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4*>(prow + ((c ^ (r & 7)) << 4)) =
            make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      if (__any_sync(0xffffffffu, need)) {
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          tc_ld32f(tl + kColO + c * 32, x);
          tc_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) x[j] *= alpha;
          tc_st32f(tl + kColO + c * 32, x);
        }
        tc_wait_st();
      }
      // Pool slots past the row length hold stale bytes (possibly NaN): P is 0
      // there but 0 * NaN is NaN, so zero those V rows of the last tile.
      if (t == ntiles - 1) {
        const int first_bad = (int)(len - (int64_t)t * kKT);
        const int last_real = min(npages * kBS - t * kKT, kKT);
        if (first_bad < last_real) {
          if (!__all_sync(0xffffffffu, wait_or_abort(&sh->full_v[s], (t >> 1) & 1, sh, a.err))) {
            failed = true;
            continue;
          }
          unsigned char* vs = smem + kOffV + s * kTile;
          const int nchunks = (last_real - first_bad) * 16;  // rows x (2 halves x 8 chunks)
          for (int e = sw * 32 + lane; e < nchunks; e += kSoftmaxThreads) {
            const int row_k = first_bad + e / 16;
            const int rem = e % 16;
            *reinterpret_cast<uint4*>(vs + (rem >> 3) * kHalf + row_k * 128 + ((rem & 7) << 4)) =
                make_uint4(0, 0, 0, 0);
          }
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&sh->p_full);
    }
    // ---- epilogue: this thread's 64 output dims ----
    red[kRows * half + r] = l;
    named_barrier_sync(pair_bar, 64);
    const float lt = l + red[kRows * (half ^ 1) + r];
    if (!failed && ntiles > 0) {
      const bool ok = __all_sync(0xffffffffu, wait_or_abort(&sh->pv_done, (ntiles - 1) & 1, sh, a.err));
      if (ok) {
        tc_fence_after();
        const float inv = lt > 0.f ? 1.f / lt : 0.f;
        T* orow = reinterpret_cast<T*>(a.out) + b * a.o_sb + (qo + (valid ? qi : 0)) * a.o_st + (int64_t)hq * a.o_sh +
                  half * 64;
        float o[32];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          tc_ld32f(tl + kColO + c * 32, o);
          tc_wait_ld();
          if (valid) {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              reinterpret_cast<uint32_t*>(orow + c * 32)[j] = pack2<T>(o[2 * j] * inv, o[2 * j + 1] * inv);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tc_dealloc(tmem, kTmemCols);
  }
}

size_t smem_bytes() { return 1024 + kSmemData + sizeof(Shared) + 4 * kRows * sizeof(float); }

template <bool BF16>
int launch(const bl_prefill_args& a, cudaStream_t s) {
  static bool attr_done = false;
  if (!attr_done) {
    if (cudaFuncSetAttribute(prefill_tc5_kernel<BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem_bytes()) != cudaSuccess) {
      set_error("prefill: cudaFuncSetAttribute failed");
      return BL_ERR_LAUNCH;
    }
    attr_done = true;
  }
  const uint64_t rows = (uint64_t)a.kv.num_layers * a.kv.num_blocks * a.kv.num_kv_heads * kBS;
  CUtensorMap kmap, vmap;
  if (!get_pool_tmap(a.kv.k_pool, rows, a.kv.dtype, &kmap) || !get_pool_tmap(a.kv.v_pool, rows, a.kv.dtype, &vmap))
    return BL_ERR_LAUNCH;
  Args k;
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
  k.rows_total = (int32_t)rows;
  k.scale_log2 = a.scale * kLog2e;
  k.err = a.err;
  const int64_t tiles = (a.max_q_len + k.bq - 1) / k.bq;
  dim3 grid((unsigned)tiles, (unsigned)a.kv.num_kv_heads, (unsigned)a.batch);
  prefill_tc5_kernel<BF16><<<grid, kThreads, smem_bytes(), s>>>(k, kmap, vmap);
  BL_CHECK_LAUNCH("prefill_tc5_kernel");
  return BL_OK;
}

}  // namespace

int prefill_tc5_launch(const bl_prefill_args& a, cudaStream_t s) {
  const uint64_t rows = (uint64_t)a.kv.num_layers * a.kv.num_blocks * a.kv.num_kv_heads * kBS;
  BL_CHECK_ARG(rows + kBS <= (uint64_t)INT32_MAX, "bl_paged_prefill: pool has more than 2^31 rows");
  BL_CHECK_ARG(((uintptr_t)a.kv.k_pool & 15) == 0 && ((uintptr_t)a.kv.v_pool & 15) == 0,
               "bl_paged_prefill: pools must be 16-byte aligned");
  BL_CHECK_ARG(((uintptr_t)a.q & 3) == 0 && ((uintptr_t)a.out & 3) == 0 && a.q_stride_b % 2 == 0 &&
                   a.q_stride_t % 2 == 0 && a.q_stride_h % 2 == 0 && a.out_stride_b % 2 == 0 &&
                   a.out_stride_t % 2 == 0 && a.out_stride_h % 2 == 0,
               "bl_paged_prefill: q/out must be 4-byte aligned with even strides");
  if (a.kv.dtype == BL_BF16) return launch<true>(a, s);
  return launch<false>(a, s);
}

}  // namespace bl
