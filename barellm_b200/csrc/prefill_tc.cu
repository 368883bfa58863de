// Paged chunked-prefill attention on 5th-generation tensor cores (tcgen05 +
// tensor memory), bf16 / fp16, head_dim 128, block_size 16, GQA group G in
// {1, 2, 4, 8}.
//
// A CTA owns one 128-row MMA tile of score rows = (128 / G) query tokens x
// the G query heads that share one KV head (head-major rows), and walks the
// keys in tiles of 128 (8 pages).  Tensor memory (512 columns) holds two S
// buffers, the O accumulator and two P buffers:
//   S0 0..127, S1 128..255, O 256..383, P0 384..447, P1 448..511,
// so no step waits for the one before it to release its columns: S(t+1) is
// computed into the other S buffer while the softmax of tile t runs, and
// P(t) goes to its own columns, where the P V MMA reads it as its A operand.
// Warp roles (8 warps, 1 CTA per SM):
//   warp 0      K producer (one lane): the 8 pages of key tile t as 2-D TMA
//               boxes (64 x 16, 128-byte swizzle) into a 3-stage K ring; a
//               page past the row's last page is read at an out-of-range row
//               coordinate, which TMA fills with zeros.
//   warp 1      V producer: the V pages of tile t into a 3-stage V ring, as
//               the same TMA boxes (lane 0), except the page holding the
//               row's last key when the row ends inside it: the 32 lanes copy
//               it with 16-byte cp.async, zero-filling the slots past the row
//               length (src-size 0), so stale pool bytes never reach P V.
//               TMA bytes and the lanes' cp.async arrivals complete the
//               stage's mbarrier together.
//   warp 2      TMEM owner and, on one lane, the MMA issuer: per key tile t it
//               issues S(t) = Q K_t^T into S[t%2] (once the softmax has read
//               S(t-2) out of it), then O += P(t-1) V_{t-1} (once P(t-1) is
//               written), so the tensor pipe computes S(t+1) and P V while
//               the softmax of tile t runs.  (Warp 3 has no role.)
//   warps 4..7  softmax, one thread per score row (= TMEM lane): S row read
//               from TMEM once into registers (bottom-right causal mask, row
//               max in log2 units), exponentiated and written as packed
//               bf16/fp16 P into P[t%2] (after the P V that last read that
//               buffer completed); a lazy rescale touches O only when the
//               running max grows by more than 2^8 (after the previous P V
//               has landed in O).  Epilogue: O / l from TMEM to global.
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
constexpr int kRows = 128;               // score rows per CTA (one MMA tile, M)
constexpr int kKStages = 3;              // K: 3 x 32 KB
constexpr int kVStages = 3;              // V: 3 x 32 KB
constexpr int kKWarp = 0;
constexpr int kVWarp = 1;
constexpr int kMmaWarp = 2;
constexpr int kSoftmaxWarp0 = 4;         // warps 4..7: TMEM lane quadrants 0..3
constexpr int kThreads = 256;
constexpr int kHalf = 128 * 128;         // 16 KB: 128 rows x 128 B (64 elements of D or K)
constexpr int kTile = 2 * kHalf;         // 32 KB
constexpr int kOffQ = 0;                         // Q: one 32 KB tile
constexpr int kOffK = kTile;                     // + s * kTile
constexpr int kOffV = kOffK + kKStages * kTile;  // + s * kTile
constexpr int kSmemData = kOffV + kVStages * kTile;  // 224 KB
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0;                    // + (t % 2) * 128
constexpr uint32_t kColO = 256;
constexpr uint32_t kColP = 384;                  // + (t % 2) * 64
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;        // log2 units

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
  int32_t rows_total;  // rows of the K tensor map: an out-of-range row coordinate
  int32_t hkv, g, bq;  // bq = query tokens per CTA = kRows / g
  int64_t num_blocks, layer_row0, max_q;
  float scale_log2;
  int32_t* err;
};

struct Shared {
  uint64_t full_k[kKStages], full_v[kVStages], empty_k[kKStages], empty_v[kVStages];
  uint64_t s_full[2], s_free[2], p_full[2], pv_done[2], q_full, mma_done;
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
      mbar_init(&sh->s_free[x], kRows);  // one arrival per softmax thread
      mbar_init(&sh->p_full[x], kRows);
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

  if (warp == kKWarp || warp == kVWarp) {
    // ------------------------------ producers ------------------------------
    const int64_t brow = a.row_ids ? (int64_t)a.row_ids[b] : b;
    const int32_t* bt = a.block_tables + brow * a.bt_stride;
    if (warp == kKWarp) {
      // K: one TMA per page half (64 x 16 box, 128-byte swizzle); pages past
      // the row's last page come from an out-of-range row, which TMA fills
      // with zeros (stale rows inside the last page are masked out of S).
      if (lane == 0) {
        if (table_short) raise_dev(a.err, BL_DEVERR_TABLE);
        prefetch_tensormap(&kmap);
        int issued = 0;
        for (int t = 0; t < ntiles; ++t) {
          const int s = t % kKStages;
          if (!wait_or_abort(&sh->empty_k[s], ((t / kKStages) & 1) ^ 1, sh, a.err)) break;
          unsigned char* dst = smem + kOffK + s * kTile;
          mbar_arrive_expect_tx(&sh->full_k[s], kTile);
#pragma unroll 1
          for (int p = 0; p < kPPT; ++p) {
            const int lb = t * kPPT + p;
            int32_t y = a.rows_total;
            if (lb < npages) {
              const int64_t phys = bt[lb];
              if (phys < 0 || phys >= a.num_blocks)
                raise_dev(a.err, BL_DEVERR_BLOCK_ID);
              else
                y = (int32_t)(a.layer_row0 + (phys * a.hkv + h) * kBS);
            }
            tma_load_2d(dst + p * kBS * 128, &kmap, &sh->full_k[s], 0, y);
            tma_load_2d(dst + kHalf + p * kBS * 128, &kmap, &sh->full_k[s], 64, y);
          }
          ++issued;
        }
        // drain: the K copies in flight land before the CTA can exit
        for (int s = 0; s < kKStages && s < issued; ++s) {
          const int last = s + ((issued - 1 - s) / kKStages) * kKStages;
          if (!mbar_wait(&sh->full_k[s], (last / kKStages) & 1)) raise_dev(a.err, BL_DEVERR_TIMEOUT);
        }
      }
    } else {
      // V: the tile's pages as 2-D TMA boxes like K (lane 0), except the page
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
        const int s = j % kVStages;
        if (!__all_sync(0xffffffffu, wait_or_abort(&sh->empty_v[s], ((j / kVStages) & 1) ^ 1, sh, a.err))) break;
        unsigned char* stage = smem + kOffV + s * kTile;
        const int64_t first = (int64_t)j * kPPT;
        const int pp = (part_lb >= first && part_lb < first + kPPT && part_lb < npages) ? (int)(part_lb - first) : -1;
        if (lane == 0) {
          mbar_arrive_expect_tx(&sh->full_v[s], (pp >= 0 ? kPPT - 1 : kPPT) * 2 * kBS * 128);
#pragma unroll 1
          for (int p = 0; p < kPPT; ++p) {
            if (p == pp) continue;
            const int lb = j * kPPT + p;
            int32_t y = a.rows_total;  // out of range: zeros
            if (lb < npages) {
              const int64_t phys = bt[lb];
              if (phys >= 0 && phys < a.num_blocks) y = (int32_t)(a.layer_row0 + (phys * a.hkv + h) * kBS);
            }
            tma_load_2d(stage + p * kBS * 128, &vmap, &sh->full_v[s], 0, y);
            tma_load_2d(stage + kHalf + p * kBS * 128, &vmap, &sh->full_v[s], 64, y);
          }
        }
        if (pp >= 0) {
          // 16 rows x 16 chunks of 16 bytes, eight per lane, in the 128-byte
          // swizzled layout the TMA boxes produce
          const int64_t lb = first + pp;
          const int64_t ph = bt[lb];
          const bool okp = ph >= 0 && ph < a.num_blocks;
#pragma unroll
          for (int e = lane; e < kBS * 16; e += 32) {
            const int r = e >> 4, cc = e & 15;
            const uint32_t bytes = (okp && lb * kBS + r < len) ? 16u : 0u;
            const uint16_t* src =
                a.v_pool + ((a.layer_row0 + ((okp ? ph : 0) * a.hkv + h) * kBS + r) * kD + cc * 8);
            const uint32_t dst =
                smem_u32(stage + (cc >> 3) * kHalf + (pp * kBS + r) * 128 + (((cc & 7) ^ (r & 7)) << 4));
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
      const uint32_t idesc_s = umma_idesc_f16(kRows, kKT, BF16, false);
      const uint32_t idesc_o = umma_idesc_f16(kRows, kD, BF16, true);
      // Shared-memory descriptors are built once; an MMA's operand address is
      // the base descriptor plus its (16-byte unit) offset.
      const uint64_t dq = umma_desc_sw128(smem_u32(smem + kOffQ), 16, 1024);
      const uint64_t dk0 = umma_desc_sw128(smem_u32(smem + kOffK), 16, 1024);
      const uint64_t dv0 = umma_desc_sw128(smem_u32(smem + kOffV), kHalf, 1024);
      const uint64_t dstage = (uint64_t)(kTile >> 4);  // one stage, in 16-byte units
      // A stage's copies land through the async proxy (TMA) or, for V's
      // partial page, through cp.async; after its mbarrier completes, a proxy
      // fence orders them before the tensor core's reads.
      auto landed = [&](uint64_t* full, uint32_t parity) -> bool {
        if (!wait_or_abort(full, parity, sh, a.err)) return false;
        fence_proxy_async_smem();
        return true;
      };
      // S(t) = Q K_t^T into S[t%2], once the softmax has read S(t-2) from it
      auto qk = [&](int t) -> bool {
        if (!landed(&sh->full_k[t % kKStages], (t / kKStages) & 1)) return false;
        if (t >= 2 && !wait_or_abort(&sh->s_free[t & 1], ((t - 2) >> 1) & 1, sh, a.err)) return false;
        tc_fence_after();
        const uint64_t dk = dk0 + (uint64_t)(t % kKStages) * dstage;
        const uint32_t d = tmem + kColS + (t & 1) * 128;
#pragma unroll
        for (int ks = 0; ks < kD / 16; ++ks) {
          const uint32_t off = ((ks >> 2) * kHalf + (ks & 3) * 32) >> 4;
          tc_mma_ss(d, dq + off, dk + off, idesc_s, ks > 0 ? 1u : 0u);
        }
        tc_commit(&sh->s_full[t & 1]);
        tc_commit(&sh->empty_k[t % kKStages]);
        return true;
      };
      // O += P(j) V_j, once P(j) is written (P in TMEM, the A operand)
      auto pv = [&](int j) -> bool {
        if (!wait_or_abort(&sh->p_full[j & 1], (j >> 1) & 1, sh, a.err)) return false;
        if (!landed(&sh->full_v[j % kVStages], (j / kVStages) & 1)) return false;
        tc_fence_after();
        const uint64_t dv = dv0 + (uint64_t)(j % kVStages) * dstage;
        const uint32_t d = tmem + kColO, pa = tmem + kColP + (j & 1) * 64;
        tc_mma_ts(d, pa, dv, idesc_o, j > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 1; kk < kKT / 16; ++kk) tc_mma_ts(d, pa + kk * 8, dv + ((kk * 2048) >> 4), idesc_o, 1u);
        tc_commit(&sh->pv_done[j & 1]);
        tc_commit(&sh->empty_v[j % kVStages]);
        return true;
      };
      // Issue order: S(0); then for t >= 1: S(t), P V(t-1); finally P V(last).
      bool ok = wait_or_abort(&sh->q_full, 0, sh, a.err);
      if (ok) {
        tc_fence_after();
        ok = qk(0);
      }
      for (int t = 1; t < ntiles && ok; ++t) ok = qk(t) && pv(t - 1);
      if (ok) ok = pv(ntiles - 1);
      // every MMA issued here has finished before the CTA tears down
      tc_commit(&sh->mma_done);
      if (!mbar_wait(&sh->mma_done, 0)) raise_dev(a.err, BL_DEVERR_TIMEOUT);
    }
  } else if (warp >= kSoftmaxWarp0) {
    // ------------------------------ softmax ------------------------------
    const int grp = warp & 3;             // TMEM lane quadrant
    const int r = 32 * grp + lane;        // row within the tile == TMEM lane
    const uint32_t tl = tmem + ((uint32_t)(32 * grp) << 16);
    const int hd = r / a.bq;
    const int tok = r - hd * a.bq;
    const int64_t qi = q0 + tok;
    const bool valid = qi < nq;
    const int hq = h * a.g + hd;
    const int64_t lim = prefix + qi;  // inclusive key limit
    // Q rows -> shared memory (K-major, 128-byte swizzle).  With 16-byte
    // aligned rows the 128 softmax threads copy 16-byte chunks (a warp reads
    // two whole 256-byte rows at a time); rows past the chunk end are zeros.
    if (a.q_vec16) {
      const int i = (warp - kSoftmaxWarp0) * 32 + lane;  // 0..127
      const int qc = i & 15;
#pragma unroll 4
      for (int k = 0; k < 16; ++k) {
        const int row = (i >> 4) + 8 * k;
        const int rhd = row / a.bq, rtok = row - rhd * a.bq;
        const int64_t rqi = q0 + rtok;
        const bool rvalid = rqi < nq;
        const T* src = reinterpret_cast<const T*>(a.q) + b * a.q_sb + (qo + (rvalid ? rqi : 0)) * a.q_st +
                       (int64_t)(h * a.g + rhd) * a.q_sh + qc * 8;
        const uint32_t dst =
            smem_u32(smem + kOffQ + (qc >> 3) * kHalf + row * 128 + (((qc & 7) ^ (row & 7)) << 4));
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(rvalid ? 16u : 0u)
                     : "memory");
      }
      asm volatile("cp.async.wait_all;" ::: "memory");
    } else {
      const T* qrow = reinterpret_cast<const T*>(a.q) + b * a.q_sb + (qo + (valid ? qi : 0)) * a.q_st +
                      (int64_t)hq * a.q_sh;
      unsigned char* qs = smem + kOffQ + r * 128;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        uint4 v = make_uint4(0, 0, 0, 0);
        if (valid) {
          const uint32_t* src = reinterpret_cast<const uint32_t*>(qrow + c * 8);
          v = make_uint4(src[0], src[1], src[2], src[3]);
        }
        *reinterpret_cast<uint4*>(qs + (c >> 3) * kHalf + (((c & 7) ^ (r & 7)) << 4)) = v;
      }
    }
    fence_proxy_async_smem();
    mbar_arrive(&sh->q_full);

    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int t = 0; t < ntiles; ++t) {
      const int x = t & 1;
      ok = __all_sync(0xffffffffu, wait_or_abort(&sh->s_full[x], (t >> 1) & 1, sh, a.err));
      if (!ok) break;
      tc_fence_after();
      const int64_t k0 = (int64_t)t * kKT;
      // the whole S row in registers: one TMEM read per tile, after which
      // S[x] is free for S(t+2)
      float v[kKT];
#pragma unroll
      for (int c = 0; c < kKT / 32; ++c) tc_ld32f(tl + kColS + x * 128 + c * 32, v + c * 32);
      tc_wait_ld();
      reg_fence<kKT>(v);
      tc_fence_before();
      mbar_arrive(&sh->s_free[x]);
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
      // P[x] was last read by P V(t-2)
      if (t >= 2) {
        ok = __all_sync(0xffffffffu, wait_or_abort(&sh->pv_done[x], ((t - 2) >> 1) & 1, sh, a.err));
        if (!ok) break;
      }
      // lazy rescale of O, once P V(t-1) has landed in it; rare once the
      // running max has settled
      if (__any_sync(0xffffffffu, need)) {
        ok = __all_sync(0xffffffffu, wait_or_abort(&sh->pv_done[x ^ 1], ((t - 1) >> 1) & 1, sh, a.err));
        if (!ok) break;
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          float o[32];
          tc_ld32f(tl + kColO + c * 32, o);
          tc_wait_ld();
          reg_fence<32>(o);
#pragma unroll
          for (int j = 0; j < 32; ++j) o[j] *= alpha;
          tc_st32f(tl + kColO + c * 32, o);
        }
      }
      tc_fence_after();
      // P = exp2(s * scale - m), packed two per column into P[x]
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
        tc_st16(tl + kColP + x * 64 + c * 16, pk);
      }
      const float rs = (rp[0] + rp[1]) + (rp[2] + rp[3]);
      tc_wait_st();
      l = l * alpha + rs;
      tc_fence_before();
      mbar_arrive(&sh->p_full[x]);
    }
    // ---- epilogue ----
    if (ok && ntiles > 0) {
      const int j = ntiles - 1;
      ok = __all_sync(0xffffffffu, wait_or_abort(&sh->pv_done[j & 1], (j >> 1) & 1, sh, a.err));
      if (ok) {
        tc_fence_after();
        const float inv = l > 0.f ? 1.f / l : 0.f;
        T* orow = reinterpret_cast<T*>(a.out) + b * a.o_sb + (qo + (valid ? qi : 0)) * a.o_st + (int64_t)hq * a.o_sh;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float o[32];
          tc_ld32f(tl + kColO + c * 32, o);
          tc_wait_ld();
          reg_fence<32>(o);
          if (valid) {
#pragma unroll
            for (int j2 = 0; j2 < 16; ++j2)
              reinterpret_cast<uint32_t*>(orow + c * 32)[j2] = pack2<T>(o[2 * j2] * inv, o[2 * j2 + 1] * inv);
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
  if (!get_pool_tmap(a.kv.k_pool, rows, a.kv.dtype, &kmap) || !get_pool_tmap(a.kv.v_pool, rows, a.kv.dtype, &vmap))
    return BL_ERR_LAUNCH;
  k.rows_total = (int32_t)rows;
  k.q_vec16 = ((uintptr_t)a.q % 16 == 0) && a.q_stride_b % 8 == 0 && a.q_stride_t % 8 == 0 && a.q_stride_h % 8 == 0;
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
