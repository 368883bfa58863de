// Paged chunked-prefill attention on 5th-generation tensor cores (tcgen05 +
// tensor memory), bf16 / fp16, head_dim 128, block_size 16, GQA group G in
// {1, 2, 4, 8}.
//
// A CTA owns 256 score rows = (256 / G) query tokens x the G query heads that
// share one KV head, as two 128-row tiles A and B (head-major rows, so for
// G >= 2 both tiles cover the same tokens and need the same keys).  Every K/V
// page is fetched once for 256 rows, which halves the K/V bytes per flop of a
// 128-row tile; keys are consumed in tiles of 128 (8 pages).  Warp roles (12 warps):
//   warp 0      K producer: the 8 pages of key tile t, one TMA box per whole
//               4 KB page (a 4-D view of the pool, 128-byte swizzle; lanes
//               0..7 one page each), into a 2-stage K ring; a page past the
//               row's last page is read at an out-of-range coordinate, which
//               TMA fills with zeros.  A page lands as [8-row group][half]
//               [8 rows][128 B], so a tile is an MMA operand whose 8-key groups
//               are 2 KB apart and whose two 64-element halves are 1 KB apart.
//   warp 1      V producer: the V pages of tile t-1 into a 3-stage V ring, as
//               the same TMA boxes (lanes 0..7), except the page holding the
//               row's last key when the row ends inside it: the 32 lanes copy
//               it with 16-byte cp.async, zero-filling the slots past the row
//               length (src-size 0), so stale pool bytes never reach P V.
//               TMA bytes and the lanes' cp.async arrivals complete the
//               stage's mbarrier together.  (Warp 2 has no role.)
//               Both producer warps hold the row's block-table entries 32 at
//               a time across their lanes and read the next 32 while using
//               the current ones: a dependent table read per page (eight per
//               tile, one after another) had held the producers to ~3.5 k
//               cycles per tile.
//   warp 3      TMEM owner (512 columns: S_A 0..127, S_B 128..255, O_A 256..383,
//               O_B 384..511) and, on one lane, the MMA issuer.  Per key tile t
//               it issues O_A += P_A V_{t-1}, S_A = Q_A K_t^T, O_B += P_B V_{t-1},
//               S_B = Q_B K_t^T, so one tile's softmax runs while the tensor
//               pipe works on the other tile.  S_X(t) is issued right behind
//               the P V that reads P_X from S_X's columns, without waiting for
//               it: the tensor pipe runs one thread's MMAs in issue order (the
//               ordering CUTLASS's Blackwell FMHA mainloop also relies on), so
//               the overwrite follows the read.
//   warps 4..7  softmax of tile A, warps 8..11 of tile B: one thread per score
//               row (= TMEM lane).  The S row is read from TMEM once into
//               registers (bottom-right causal mask, row max in log2 units),
//               exponentiated and written back as packed bf16/fp16 P over the
//               first 64 S columns, where the P V MMA reads it as its A
//               operand; a lazy rescale touches O only when the running max
//               grows by more than 2^8.  Epilogue: O / l from TMEM, staged in
//               Q's shared memory and written back as whole 256-byte rows.
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
constexpr int kTileRows = 128;           // rows per MMA tile (M)
constexpr int kRows = 2 * kTileRows;     // score rows per CTA
constexpr int kKStages = 2;             // K: 2 x 32 KB (S of tile t+1 is issued after P V of t-1)
constexpr int kVStages = 3;             // V: 3 x 32 KB (V is read last, by P V)
constexpr int kMmaWarp = 3;
constexpr int kSoftmaxWarp0 = 4;
constexpr int kThreads = 384;            // 3 producer warps, MMA warp, 2 x 4 softmax warps
constexpr int kHalf = 128 * 128;         // 16 KB: a Q tile's 128 rows x 128 B (64 elements of D)
constexpr int kTile = 2 * kHalf;         // 32 KB
constexpr int kPage = kBS * kD * 2;      // 4 KB: one page in a K / V stage
constexpr int kGroup = 2048;             // 8 key rows (both halves) in a K / V stage
constexpr int kOffQ = 0;                        // + X * kTile
constexpr int kOffK = 2 * kTile;                // + s * kTile
constexpr int kOffV = kOffK + kKStages * kTile;  // + s * kTile
constexpr int kSmemData = kOffV + kVStages * kTile;  // 224 KB
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0;                   // + X * 128 (P_X aliases the first 64 columns)
constexpr uint32_t kColO = 256;                 // + X * 128
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
  const uint16_t* k_pool;
  const uint16_t* v_pool;
  int32_t q_vec16;  // q rows start on 16-byte boundaries (pointer and strides)
  int32_t o_vec16;  // out rows start on 16-byte boundaries (pointer and strides)
  int32_t rows_total;  // rows of the K tensor map: an out-of-range row coordinate
  int32_t hkv, g, bq;  // bq = query tokens per CTA = kRows / g
  int64_t num_blocks, layer_row0, max_q;
  float scale_log2;
  int32_t* err;
};

struct Shared {
  uint64_t full_k[kKStages], full_v[kVStages], empty_k[kKStages], empty_v[kVStages];
  uint64_t s_full[2], p_full[2], pv_done[2], q_full, mma_done;
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
    prefill_tc_kernel(const Args a, const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap) {
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Shared* sh = reinterpret_cast<Shared*>(smem + kSmemData);

  // ---- which rows: heaviest query tiles first ----
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
    for (int s = 0; s < kKStages; ++s) {
      mbar_init(&sh->full_k[s], 1);
      mbar_init(&sh->empty_k[s], 1);
    }
    for (int s = 0; s < kVStages; ++s) {
      mbar_init(&sh->full_v[s], 1 + 32);  // V lane 0's arrive.expect_tx + one cp.async arrival per lane
      mbar_init(&sh->empty_v[s], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&sh->s_full[x], 1);
      mbar_init(&sh->p_full[x], kTileRows);
      mbar_init(&sh->pv_done[x], 1);
    }
    mbar_init(&sh->q_full, kRows);
    mbar_init(&sh->mma_done, 1);
    sh->abort = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) tc_alloc(&sh->tmem_base, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;

  if (warp < kMmaWarp) {
    // ------------------------------ producers ------------------------------
    const int64_t brow = a.row_ids ? (int64_t)a.row_ids[b] : b;
    const int32_t* bt = a.block_tables + brow * a.bt_stride;
    // The row's block-table entries reach each producer warp 32 at a time
    // (four key tiles), lane i holding page 32k + i, and the next 32 are read
    // while the current ones are in use: a producer never waits on a
    // dependent table read per page (eight of them in a row cost more than a
    // whole tile's MMAs).
    auto bt_at = [&](int lb) -> int32_t { return lb < npages ? bt[lb] : -1; };
    int32_t win_cur = bt_at(lane), win_nxt = bt_at(32 + lane);
    auto advance = [&](int t) {
      if (t > 0 && (t & 3) == 0) {
        win_cur = win_nxt;
        win_nxt = bt_at((t + 4) * kPPT + lane);
      }
    };
    // the pool coordinate of page lb (held by this lane), or out of range
    auto page_w = [&](int lb, int32_t phys, bool flag) -> int32_t {
      if (lb >= npages) return a.rows_total / 8;  // past the row: zeros
      if (phys < 0 || phys >= a.num_blocks) {
        if (flag) raise_dev(a.err, BL_DEVERR_BLOCK_ID);
        return a.rows_total / 8;
      }
      return (int32_t)((a.layer_row0 + ((int64_t)phys * a.hkv + h) * kBS) / 8);
    };
    if (warp == 0) {
      // K: one TMA box per page, lanes 0..7 one page each; pages past the
      // row's last page come from an out-of-range coordinate, which TMA fills
      // with zeros (stale rows inside the last page are masked out of S).
      if (lane == 0) {
        if (table_short) raise_dev(a.err, BL_DEVERR_TABLE);
        prefetch_tensormap(&kmap);
      }
      int issued = 0;
      for (int t = 0; t < ntiles; ++t) {
        advance(t);
        const int s = t % kKStages;
        if (!__all_sync(0xffffffffu, wait_or_abort(&sh->empty_k[s], ((t / kKStages) & 1) ^ 1, sh, a.err))) break;
        const int32_t phys = __shfl_sync(0xffffffffu, win_cur, (t & 3) * kPPT + (lane & (kPPT - 1)));
        unsigned char* dst = smem + kOffK + s * kTile;
        if (lane == 0) mbar_arrive_expect_tx(&sh->full_k[s], kTile);
        __syncwarp();
        if (lane < kPPT) {
          const int32_t w = page_w(t * kPPT + lane, phys, true);
          tma_load_4d(dst + lane * kPage, &kmap, &sh->full_k[s], 0, 0, 0, w);
        }
        ++issued;
      }
      // drain: the K copies in flight land before the CTA can exit
      if (lane == 0) {
        for (int s = 0; s < kKStages && s < issued; ++s) {
          const int last = s + ((issued - 1 - s) / kKStages) * kKStages;
          if (!mbar_wait(&sh->full_k[s], (last / kKStages) & 1)) raise_dev(a.err, BL_DEVERR_TIMEOUT);
        }
      }
    } else if (warp == 1) {
      // V: the tile's pages as TMA boxes like K (lanes 0..7), except the page
      // holding the row's last key when the row ends inside it.  Its slots
      // past the length may hold stale pool bytes (NaN included), which P V
      // would turn into NaN even where P = 0, so the warp copies that page
      // with 16-byte cp.async and zero-fills those slots (src-size 0).  Both
      // land on the stage's mbarrier: lane 0's arrive.expect_tx for the TMA
      // bytes plus one cp.async arrival per lane, every tile.
      const int64_t part_lb = (len % kBS) ? (len - 1) / kBS : -1;
      if (lane == 0) prefetch_tensormap(&vmap);
      int issued = 0;
      for (int j = 0; j < ntiles; ++j) {
        advance(j);
        const int s = j % kVStages;
        if (!__all_sync(0xffffffffu, wait_or_abort(&sh->empty_v[s], ((j / kVStages) & 1) ^ 1, sh, a.err))) break;
        unsigned char* stage = smem + kOffV + s * kTile;
        const int64_t first = (int64_t)j * kPPT;
        const int pp = (part_lb >= first && part_lb < first + kPPT && part_lb < npages) ? (int)(part_lb - first) : -1;
        const int32_t phys = __shfl_sync(0xffffffffu, win_cur, (j & 3) * kPPT + (lane & (kPPT - 1)));
        const int32_t ph = __shfl_sync(0xffffffffu, win_cur, (j & 3) * kPPT + (pp >= 0 ? pp : 0));
        if (lane == 0) mbar_arrive_expect_tx(&sh->full_v[s], (pp >= 0 ? kPPT - 1 : kPPT) * kPage);
        __syncwarp();
        if (lane < kPPT && lane != pp) {
          const int32_t w = page_w((int)first + lane, phys, false);
          tma_load_4d(stage + lane * kPage, &vmap, &sh->full_v[s], 0, 0, 0, w);
        }
        if (pp >= 0) {
          // 16 rows x 16 chunks of 16 bytes, eight per lane, in the layout the
          // page boxes produce: [8-row group][half][8 rows][128 B], swizzled
          const int64_t lb = first + pp;
          const bool okp = ph >= 0 && ph < a.num_blocks;
#pragma unroll
          for (int e = lane; e < kBS * 16; e += 32) {
            const int r = e >> 4, cc = e & 15;
            const uint32_t bytes = (okp && lb * kBS + r < len) ? 16u : 0u;
            const uint16_t* src =
                a.v_pool + ((a.layer_row0 + ((okp ? (int64_t)ph : 0) * a.hkv + h) * kBS + r) * kD + cc * 8);
            const uint32_t dst = smem_u32(stage + pp * kPage + (r >> 3) * kGroup + (cc >> 3) * 1024 + (r & 7) * 128 +
                                          (((cc & 7) ^ (r & 7)) << 4));
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
          }
        }
        asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(&sh->full_v[s])) : "memory");
        ++issued;
      }
      // drain: the V copies in flight land before the CTA can exit
      if (lane == 0) {
        for (int s = 0; s < kVStages && s < issued; ++s) {
          const int last = s + ((issued - 1 - s) / kVStages) * kVStages;
          if (!mbar_wait(&sh->full_v[s], (last / kVStages) & 1)) raise_dev(a.err, BL_DEVERR_TIMEOUT);
        }
      }
    }
    // every copy this thread issued lands before the CTA can exit
    asm volatile("cp.async.wait_all;" ::: "memory");
  } else if (warp == kMmaWarp) {
    // ------------------------------ MMA issuer ------------------------------
    if (lane == 0) {
      const uint32_t idesc_s = umma_idesc_f16(kTileRows, kKT, BF16, false);
      const uint32_t idesc_o = umma_idesc_f16(kTileRows, kD, BF16, true);
      // O_X += P_X V_j (P_X in S_X's TMEM columns)
      // Shared-memory descriptors are built once; an MMA's operand address is
      // the base descriptor plus its (16-byte unit) offset, so the single
      // issuing thread spends a few instructions per MMA (a 128 x 128 x 16 step
      // takes 64 cycles on the tensor pipe, less than rebuilding descriptors).
      const uint64_t dq0 = umma_desc_sw128(smem_u32(smem + kOffQ), 16, 1024);
      const uint64_t dq1 = umma_desc_sw128(smem_u32(smem + kOffQ + kTile), 16, 1024);
      const uint64_t dk0 = umma_desc_sw128(smem_u32(smem + kOffK), 16, kGroup);  // 8-key groups kGroup apart
      const uint64_t dk_stride = (uint64_t)(kTile >> 4);  // one K stage, in 16-byte units
      const uint64_t dv0 = umma_desc_sw128(smem_u32(smem + kOffV), 1024, kGroup);  // MN-major: halves 1 KB apart
      // O_X += P_X V_j (P_X in S_X's TMEM columns)
      auto pv = [&](int x, int j) -> bool {
        if (!wait_or_abort(&sh->p_full[x], j & 1, sh, a.err)) return false;
        tc_fence_after();
        const uint64_t dv = dv0 + (uint64_t)(j % kVStages) * (uint64_t)(kTile >> 4);
        const uint32_t d = tmem + kColO + x * 128, pa = tmem + kColS + x * 128;
        tc_mma_ts(d, pa, dv, idesc_o, j > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 1; kk < kKT / 16; ++kk) tc_mma_ts(d, pa + kk * 8, dv + ((kk * kPage) >> 4), idesc_o, 1u);
        if (j == ntiles - 1) tc_commit(&sh->pv_done[x]);  // O_X final: the epilogue's signal
        return true;
      };
      // S_X = Q_X K_t^T, queued behind the P V that last read S_X's columns
      auto qk = [&](int x, int t) -> bool {
        const uint64_t dq = x ? dq1 : dq0, dk = dk0 + (uint64_t)(t % kKStages) * dk_stride;
        const uint32_t d = tmem + kColS + x * 128;
#pragma unroll
        for (int ks = 0; ks < kD / 16; ++ks) {
          const uint32_t off = ((ks >> 2) * kHalf + (ks & 3) * 32) >> 4;
          const uint32_t koff = ((ks >> 2) * 1024 + (ks & 3) * 32) >> 4;
          tc_mma_ss(d, dq + off, dk + koff, idesc_s, ks > 0 ? 1u : 0u);
        }
        tc_commit(&sh->s_full[x]);
        return true;
      };
      // K stages are written by TMA only (the async proxy the tensor core
      // reads through); a V stage also holds the row's partial last page when
      // it ends inside that tile, written by cp.async (generic proxy): only
      // then does the issuer need a proxy fence after the stage's barrier.
      const int64_t part_lb = (len % kBS) ? (len - 1) / kBS : -1;
      auto landed_k = [&](int t) -> bool {
        return wait_or_abort(&sh->full_k[t % kKStages], (t / kKStages) & 1, sh, a.err);
      };
      auto landed_v = [&](int j) -> bool {
        if (!wait_or_abort(&sh->full_v[j % kVStages], (j / kVStages) & 1, sh, a.err)) return false;
        if (part_lb >= (int64_t)j * kPPT && part_lb < (int64_t)j * kPPT + kPPT) fence_proxy_async_smem();
        return true;
      };
      // Issue order per key tile t >= 1:  PV_A(t-1), S_A(t), PV_B(t-1), S_B(t),
      // so tile A's softmax of t runs while the tensor pipe works on tile B.
      bool ok = wait_or_abort(&sh->q_full, 0, sh, a.err);
      if (ok) tc_fence_after();
      if (ok && ntiles > 0) {
        ok = landed_k(0) && qk(0, 0) && qk(1, 0);
        if (ok) tc_commit(&sh->empty_k[0]);
      }
      for (int t = 1; t < ntiles && ok; ++t) {
        const int j = t - 1;
        ok = landed_v(j) && landed_k(t) && pv(0, j) && qk(0, t) && pv(1, j);
        if (!ok) break;
        tc_commit(&sh->empty_v[j % kVStages]);
        if (!(ok = qk(1, t))) break;
        tc_commit(&sh->empty_k[t % kKStages]);
      }
      if (ok && ntiles > 0) {
        const int j = ntiles - 1;
        ok = landed_v(j) && pv(0, j) && pv(1, j);
      }
      // every MMA issued here has finished before the CTA tears down
      tc_commit(&sh->mma_done);
      if (!mbar_wait(&sh->mma_done, 0)) raise_dev(a.err, BL_DEVERR_TIMEOUT);
    }
  } else {
    // ------------------------------ softmax ------------------------------
    const int x = (warp - kSoftmaxWarp0) >> 2;  // tile: 0 = A, 1 = B
    const int grp = warp & 3;             // TMEM lane group
    const int tr = 32 * grp + lane;       // row within the tile == TMEM lane
    const int r = x * kTileRows + tr;     // row within the CTA
    const uint32_t tl = tmem + ((uint32_t)(32 * grp) << 16);
    const uint32_t sc = kColS + x * 128, oc = kColO + x * 128;
    const int hd = r / a.bq;
    const int tok = r - hd * a.bq;
    const int64_t qi = q0 + tok;
    const bool valid = qi < nq;
    const int hq = h * a.g + hd;
    const int64_t lim = prefix + qi;  // inclusive key limit
    // Q rows -> shared memory (K-major, 128-byte swizzle).  With 16-byte
    // aligned rows the 256 softmax threads copy 16-byte chunks (a warp reads
    // two whole 256-byte rows at a time); rows past the chunk end are zeros.
    if (a.q_vec16) {
      const int i = (warp - kSoftmaxWarp0) * 32 + lane;  // 0..255
      const int qc = i & 15;
#pragma unroll 4
      for (int k = 0; k < 16; ++k) {
        const int row = (i >> 4) + 16 * k;
        const int rhd = row / a.bq, rtok = row - rhd * a.bq;
        const int64_t rqi = q0 + rtok;
        const bool rvalid = rqi < nq;
        const T* src = reinterpret_cast<const T*>(a.q) + b * a.q_sb + (qo + (rvalid ? rqi : 0)) * a.q_st +
                       (int64_t)(h * a.g + rhd) * a.q_sh + qc * 8;
        const int rt = row & (kTileRows - 1);
        const uint32_t dst = smem_u32(smem + kOffQ + (row >> 7) * kTile + (qc >> 3) * kHalf + rt * 128 +
                                      (((qc & 7) ^ (rt & 7)) << 4));
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(rvalid ? 16u : 0u)
                     : "memory");
      }
      asm volatile("cp.async.wait_all;" ::: "memory");
    } else {
      const T* qrow = reinterpret_cast<const T*>(a.q) + b * a.q_sb + (qo + (valid ? qi : 0)) * a.q_st +
                      (int64_t)hq * a.q_sh;
      unsigned char* qs = smem + kOffQ + x * kTile + tr * 128;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        uint4 v = make_uint4(0, 0, 0, 0);
        if (valid) {
          const uint32_t* src = reinterpret_cast<const uint32_t*>(qrow + c * 8);
          v = make_uint4(src[0], src[1], src[2], src[3]);
        }
        *reinterpret_cast<uint4*>(qs + (c >> 3) * kHalf + (((c & 7) ^ (tr & 7)) << 4)) = v;
      }
    }
    fence_proxy_async_smem();
    mbar_arrive(&sh->q_full);

    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int t = 0; t < ntiles; ++t) {
      ok = __all_sync(0xffffffffu, wait_or_abort(&sh->s_full[x], t & 1, sh, a.err));
      if (!ok) break;
      tc_fence_after();
      const int64_t k0 = (int64_t)t * kKT;
      // the whole S row in registers: one TMEM read per tile
      float v[kKT];
#pragma unroll
      for (int c = 0; c < kKT / 32; ++c) tc_ld32f(tl + sc + c * 32, v + c * 32);
      tc_wait_ld();
      reg_fence<kKT>(v);
      // bottom-right causal mask: keys past `lim` drop out (only tiles that
      // cross the diagonal or the chunk end take this branch)
      const int64_t lim_rel64 = lim - k0;
      if (__any_sync(0xffffffffu, lim_rel64 < kKT - 1)) {
        const int lim_rel = lim_rel64 < -1 ? -1 : (int)lim_rel64;
#pragma unroll
        for (int j = 0; j < kKT; ++j) v[j] = j > lim_rel ? -INFINITY : v[j];
      }
      // row max of the raw scores (the scale is positive), eight partial chains
      float mp[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mp[i] = v[i];
#pragma unroll
      for (int j = 8; j < kKT; ++j) mp[j & 7] = fmaxf(mp[j & 7], v[j]);
      const float mt = fmaxf(fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])),
                             fmaxf(fmaxf(mp[4], mp[5]), fmaxf(mp[6], mp[7]))) * a.scale_log2;
      const float m_new = fmaxf(m_used, mt);
      const bool need = (t > 0) && (m_new > m_used + kRescaleThreshold);
      const float alpha = need ? fast_exp2(m_used - m_new) : 1.f;
      if (need || t == 0) m_used = m_new;
      const float ms = (m_used == -INFINITY) ? 0.f : m_used;
      // P = exp2(s * scale - m), packed two per column over S's first 64
      // columns (S is already in registers)
      float rp[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < kKT / 32; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float p0 = fast_exp2(fmaf(v[c * 32 + 2 * j], a.scale_log2, -ms));
          const float p1 = fast_exp2(fmaf(v[c * 32 + 2 * j + 1], a.scale_log2, -ms));
          rp[j & 3] += p0 + p1;
          pk[j] = pack2<T>(p0, p1);
        }
        tc_st16(tl + sc + c * 16, pk);
      }
      const float rs = (rp[0] + rp[1]) + (rp[2] + rp[3]);
      // lazy rescale of O (S_X's commit tracks every MMA issued before it, so
      // the P V that last wrote O_X has completed); rare once the running max
      // has settled
      if (__any_sync(0xffffffffu, need)) {
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          float o[32];
          tc_ld32f(tl + oc + c * 32, o);
          tc_wait_ld();
          reg_fence<32>(o);
#pragma unroll
          for (int j = 0; j < 32; ++j) o[j] *= alpha;
          tc_st32f(tl + oc + c * 32, o);
        }
      }
      tc_wait_st();
      l = l * alpha + rs;
      tc_fence_before();
      mbar_arrive(&sh->p_full[x]);
    }
    // ---- epilogue ----
    if (ok && ntiles > 0) {
      ok = __all_sync(0xffffffffu, wait_or_abort(&sh->pv_done[x], 0, sh, a.err));
      if (ok) {
        tc_fence_after();
        const float inv = l > 0.f ? 1.f / l : 0.f;
        if (a.o_vec16) {
          // Every S MMA finished before the last P V of either tile (they were
          // issued earlier by the same thread), so Q's shared memory is free:
          // each warp stages its 32 rows there (16-byte chunks XOR-swizzled by
          // row) and writes them back as whole 256-byte rows, two per store.
          unsigned char* stage = smem + kOffQ + x * kTile + grp * (32 * kD * 2);
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            float o[32];
            tc_ld32f(tl + oc + c * 32, o);
            tc_wait_ld();
            reg_fence<32>(o);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const int ch = c * 4 + k;
              uint4 w;
              w.x = pack2<T>(o[8 * k + 0] * inv, o[8 * k + 1] * inv);
              w.y = pack2<T>(o[8 * k + 2] * inv, o[8 * k + 3] * inv);
              w.z = pack2<T>(o[8 * k + 4] * inv, o[8 * k + 5] * inv);
              w.w = pack2<T>(o[8 * k + 6] * inv, o[8 * k + 7] * inv);
              *reinterpret_cast<uint4*>(stage + lane * 256 + ((ch ^ (lane & 7)) << 4)) = w;
            }
          }
          __syncwarp();
          const int ch = lane & 15;
#pragma unroll 4
          for (int it = 0; it < 16; ++it) {
            const int rl = 2 * it + (lane >> 4);  // row within the warp's 32
            const int rr = x * kTileRows + 32 * grp + rl;
            const int rhd = rr / a.bq;
            const int64_t rqi = q0 + (rr - rhd * a.bq);
            if (rqi < nq) {
              const uint4 w = *reinterpret_cast<const uint4*>(stage + rl * 256 + ((ch ^ (rl & 7)) << 4));
              T* dst = reinterpret_cast<T*>(a.out) + b * a.o_sb + (qo + rqi) * a.o_st + (int64_t)(h * a.g + rhd) * a.o_sh;
              *reinterpret_cast<uint4*>(dst + ch * 8) = w;
            }
          }
        } else {
          T* orow = reinterpret_cast<T*>(a.out) + b * a.o_sb + (qo + (valid ? qi : 0)) * a.o_st + (int64_t)hq * a.o_sh;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            float o[32];
            tc_ld32f(tl + oc + c * 32, o);
            tc_wait_ld();
            reg_fence<32>(o);
            if (valid) {
#pragma unroll
              for (int j = 0; j < 16; ++j)
                reinterpret_cast<uint32_t*>(orow + c * 32)[j] = pack2<T>(o[2 * j] * inv, o[2 * j + 1] * inv);
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tc_dealloc(tmem, kTmemCols);
  }
}

size_t smem_bytes() { return 1024 + kSmemData + sizeof(Shared); }

template <bool BF16>
int launch(const bl_prefill_args& a, cudaStream_t s) {
  static bool attr_done = false;
  if (!attr_done) {
    if (cudaFuncSetAttribute(prefill_tc_kernel<BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem_bytes()) != cudaSuccess) {
      set_error("prefill: cudaFuncSetAttribute failed");
      return BL_ERR_LAUNCH;
    }
    attr_done = true;
  }
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
  const uint64_t rows = (uint64_t)a.kv.num_layers * a.kv.num_blocks * a.kv.num_kv_heads * kBS;
  CUtensorMap kmap, vmap;
  if (!get_pool_page_tmap(a.kv.k_pool, rows, a.kv.dtype, &kmap) || !get_pool_page_tmap(a.kv.v_pool, rows, a.kv.dtype, &vmap))
    return BL_ERR_LAUNCH;
  k.rows_total = (int32_t)rows;
  k.q_vec16 = ((uintptr_t)a.q % 16 == 0) && a.q_stride_b % 8 == 0 && a.q_stride_t % 8 == 0 && a.q_stride_h % 8 == 0;
  k.o_vec16 = ((uintptr_t)a.out % 16 == 0) && a.out_stride_b % 8 == 0 && a.out_stride_t % 8 == 0 &&
              a.out_stride_h % 8 == 0;
  k.k_pool = static_cast<const uint16_t*>(a.kv.k_pool);
  k.v_pool = static_cast<const uint16_t*>(a.kv.v_pool);
  k.scale_log2 = a.scale * kLog2e;
  k.err = a.err;
  const int64_t tiles = (a.max_q_len + k.bq - 1) / k.bq;
  dim3 grid((unsigned)tiles, (unsigned)a.kv.num_kv_heads, (unsigned)a.batch);
  prefill_tc_kernel<BF16><<<grid, kThreads, smem_bytes(), s>>>(k, kmap, vmap);
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
