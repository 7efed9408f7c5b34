// Causal grouped-query flash attention, backward, for sm_100a.
//
// Reference semantics (duoan/mega-trading):
//   src/mega_trading/kernels/triton_attention.py:80-111 (torch backward for
//   every shape: P from the saved scores, dS = P * (dP - rowsum(dP * P)),
//   dQ = scale dS K, dK = scale dS^T Q, dV = P^T dO, GQA grads summed over
//   the query heads of a group), :134-245 and :481-747 (Triton server-shape
//   backward: P recomputed from the saved logsumexp, Delta = rowsum(O * dO)).
//
// B200 design
//   * preprocess kernel: Delta = rowsum(O * dO) and lse * log2(e) into padded
//     fp32 workspace rows (+inf past T so padded queries get P = 0); the fp32
//     dQ accumulator is zeroed with cudaMemsetAsync.
//   * main kernel: work item = one 128-key tile of one (batch, KV head).  It
//     loops over every query head of the GQA group and every causal query
//     tile (query tile >= key tile).  Persistent: one CTA per SM takes items
//     from a global work counter (zeroed by the preprocess kernel; the
//     producer warp fetches each item and passes it to the MMA and compute
//     warps through a shared-memory ring), so the CTAs stay balanced although
//     items differ 16x in work; the next item's first Q/dO tiles are
//     prefetched and its K/V load overlaps this item's last dQ drain and
//     dK/dV epilogue.  All five products are tcgen05.mma with fp32
//     accumulators in TMEM:
//         S^T  = K Q^T        cols [0,128)        (M=128 keys, N=128 queries)
//         dP^T = V dO^T       cols [128,256)
//         dV  += P^T dO       cols [256,256+D)    (accumulated over the group)
//         dK  += dS^T Q       cols [256+D,256+2D)
//         dQ   = dS K         cols [256+2D,256+3D) (M=128 queries)
//     P^T is stored (bf16/fp16 pairs) into TMEM columns [448,512) and dV
//     reads it as a TMEM A operand; dS^T is written once to a 128B-swizzled
//     shared tile that serves as the K-major A operand of dK and, read
//     MN-major, as the A operand of dQ.  Q, dO and K are consumed MN-major where they
//     act as B of a key-contracted product, so nothing is transposed.
//   * dQ partials leave the CTA through a TMA bulk tensor reduce-add (fp32)
//     from a 128B-swizzled staging tile; dK/dV never leave TMEM until the
//     group is done (no atomics for them).
//   * Warp roles: warps 0-7 = two compute warpgroups (thread = key row for
//     S/dP/dS, = query row for the dQ drain; the two groups split the query
//     columns), warp 8 = TMA producer (+ TMEM allocation), warp 9 = MMA.
//   * postprocess kernel: dQ = bf16(scale * dQacc) in the caller's layout.
//   * Every mbarrier wait is bounded (status word + early exit, no trap).
#include <cmath>
#include <type_traits>

#include "common.cuh"

namespace mt {

int make_bhtd_map(CUtensorMap* map, const void* base, int dtype, int64_t B, int64_t H, int64_t T, int64_t D,
                  const int64_t* s, int box_rows, int* swapped);
int check_attn_layout(const void* ptr, const int64_t* s, bool need);

namespace {

constexpr int kBK = 128;  // keys per CTA
constexpr int kBQ = 128;  // queries per tile
constexpr int kNQ = 3;    // Q/dO pipeline stages (loads run ~2 tiles ahead of the MMAs)
constexpr int kThreads = 320;
constexpr int kRing = 4;  // work items announced ahead by the producer warp
constexpr uint32_t kKernelId = 2;

template <int D>
struct BwdCfg {
  static constexpr int ROW_BYTES = D * 2;
  static constexpr uint32_t LAYOUT = (D == 64) ? kSwizzle128 : kSwizzle64;
  static constexpr int SBO = 8 * ROW_BYTES;
  static constexpr int TILE = 128 * ROW_BYTES;
  static constexpr int PT_BYTES = kBK * kBQ * 2;  // one P^T or dS^T tile
  static constexpr int DQ_BYTES = kBQ * D * 4;    // fp32 dQ staging (D/32 boxes of 16 KB)
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = OFF_K + TILE;
  static constexpr int OFF_Q = OFF_V + TILE;
  static constexpr int OFF_DO = OFF_Q + kNQ * TILE;
  static constexpr int OFF_DS = OFF_DO + kNQ * TILE;
  static constexpr int OFF_DQ = OFF_DS + PT_BYTES;
  static constexpr int OFF_LSE = OFF_DQ + DQ_BYTES;      // [kNQ][128] fp32
  static constexpr int OFF_DELTA = OFF_LSE + kNQ * 512;  // [kNQ][128] fp32
  static constexpr int OFF_BAR = OFF_DELTA + kNQ * 512;
  static constexpr int SMEM = OFF_BAR + 256;
  static constexpr int TMEM_COLS = 512;
  static constexpr int T_S = 0, T_DP = 128, T_DV = 256, T_DK = 256 + D, T_DQ = 256 + 2 * D;
  static constexpr int T_PT = 448;  // P^T, 16-bit pairs: A operand of dV += P^T dO
};

struct BwdParams {
  CUtensorMap tm_q, tm_k, tm_v, tm_do, tm_dq;  // tm_dq: fp32 accumulator [rows, D]
  int sw_q, sw_k, sw_v, sw_do;                 // coordinate order of each bf16 map
  const float* lse2;                           // [B*Hq*Tp] -lse * log2(e), -inf past T
  const float* delta;                          // [B*Hq*Tp]
  void* dk;
  void* dv;
  int64_t dks[4], dvs[4];
  int T, Tp, Hq, Hkv, repeats, n_tiles;
  int n_heads;  // B * Hkv
  int group;    // (batch, kv head) pairs whose key tiles are interleaved in item order
  int n_items;  // n_heads * n_tiles
  int* sched;   // work counter (next item), zero at launch
  // optional RoPE tables [T, D/2] (row stride rope_ld): dk is rotated back by
  // -theta(key) before rounding, giving the gradient of the un-rotated keys
  const void* rope_cos;
  const void* rope_sin;
  int64_t rope_ld;
  float scale_log2, scale;
  uint32_t* status;
};

__device__ __forceinline__ void tma_tile(void* dst, const CUtensorMap* map, uint64_t* bar, int t0, int h, int b,
                                         int swapped) {
  if (swapped)
    tma_load_4d(dst, map, bar, 0, h, t0, b);
  else
    tma_load_4d(dst, map, bar, 0, t0, h, b);
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// Inverse RoPE of 8 consecutive features (4 interleaved pairs starting at pair
// index i0) of position t: (e, o) -> (e cos + o sin, o cos - e sin), the
// transpose of the forward rotation, with the 16-bit tables the forward used.
template <typename T>
__device__ __forceinline__ void rope_back8(float (&g)[8], const void* cos_t, const void* sin_t, int64_t ld, int t,
                                           int i0) {
  const uint2 cr = *reinterpret_cast<const uint2*>(static_cast<const T*>(cos_t) + int64_t(t) * ld + i0);
  const uint2 sr = *reinterpret_cast<const uint2*>(static_cast<const T*>(sin_t) + int64_t(t) * ld + i0);
  const T* ce = reinterpret_cast<const T*>(&cr);
  const T* se = reinterpret_cast<const T*>(&sr);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float cs = to_f32<T>(ce[i]), sn = to_f32<T>(se[i]);
    const float e = g[2 * i], od = g[2 * i + 1];
    g[2 * i] = e * cs + od * sn;
    g[2 * i + 1] = od * cs - e * sn;
  }
}

// Write 32 consecutive query columns (col0 .. col0+31, col0 % 32 == 0) of one
// key row into a 128B-swizzled [128 rows][64 cols] x 2 K-major tile.
template <typename T>
__device__ __forceinline__ void store_row32(uint8_t* tile, int row, int col0, const float (&v)[32]) {
  uint8_t* base = tile + (col0 >> 6) * (128 * 128) + row * 128;
  const int ch0 = (col0 & 63) >> 3;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 w;
    w.x = pack2<T>(v[q * 8 + 0], v[q * 8 + 1]);
    w.y = pack2<T>(v[q * 8 + 2], v[q * 8 + 3]);
    w.z = pack2<T>(v[q * 8 + 4], v[q * 8 + 5]);
    w.w = pack2<T>(v[q * 8 + 6], v[q * 8 + 7]);
    *reinterpret_cast<uint4*>(base + (((ch0 + q) ^ (row & 7)) * 16)) = w;
  }
}

// Item order: groups of `group` (batch, kv head) pairs; inside a group the
// key tiles go heaviest (smallest index) first, cycling over the group's
// heads.  The items resident at one time then share a few heads' Q / dO tiles
// and fp32 dQ rows in L2 instead of streaming every head's.
struct BwdItem {
  int b, hk, kt;
  int n_q, n_it;  // causal query tiles per head (kt .. n_tiles-1); iterations (x repeats)
};

__device__ __forceinline__ BwdItem bwd_item(const BwdParams& p, int it) {
  BwdItem w;
  const int per_group = p.group * p.n_tiles;
  const int grp = it / per_group;
  const int rem = it - grp * per_group;
  const int g0 = grp * p.group;
  const int gsz = min(p.group, p.n_heads - g0);
  w.kt = rem / gsz;
  const int bk = g0 + (rem - w.kt * gsz);
  w.b = bk / p.Hkv;
  w.hk = bk - w.b * p.Hkv;
  w.n_q = p.n_tiles - w.kt;
  w.n_it = w.n_q * p.repeats;
  return w;
}

template <typename T, int D>
__global__ void __launch_bounds__(kThreads, 1) attn_bwd_kernel(const __grid_constant__ BwdParams p) {
  using C = BwdCfg<D>;
  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = warp_id();
  const int lane = lane_id();
  if ((smem_u32(smem) & 1023u) != 0) {
    if (threadIdx.x == 0) atomicCAS(p.status, 0u, (kKernelId << 16) | 0xFFFFu);
    return;
  }
  uint8_t* sK = smem + C::OFF_K;
  uint8_t* sV = smem + C::OFF_V;
  uint8_t* sQ = smem + C::OFF_Q;
  uint8_t* sDO = smem + C::OFF_DO;
  uint8_t* sDS = smem + C::OFF_DS;
  uint8_t* sDQ = smem + C::OFF_DQ;
  float* sLse = reinterpret_cast<float*>(smem + C::OFF_LSE);
  float* sDelta = reinterpret_cast<float*>(smem + C::OFF_DELTA);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* bar_kv = bars + 0;
  uint64_t* bar_q_full = bars + 1;           // [kNQ]
  uint64_t* bar_q_empty = bar_q_full + kNQ;  // [kNQ]
  uint64_t* bar_sd_full = bar_q_empty + kNQ;
  uint64_t* bar_sd_free = bar_sd_full + 1;
  uint64_t* bar_pds_full = bar_sd_full + 2;
  uint64_t* bar_dq_full = bar_sd_full + 3;
  uint64_t* bar_dq_free = bar_sd_full + 4;
  uint64_t* bar_done = bar_sd_full + 5;
  uint64_t* bar_pt_free = bar_sd_full + 6;  // dV of the previous tile done: P^T TMEM free
  uint64_t* bar_item = bar_sd_full + 7;     // an item's last dQ done: its K/V, dK and dV are free
  uint64_t* ring_full = bar_sd_full + 8;    // [kRing] item id published
  uint64_t* ring_empty = ring_full + kRing;  // [kRing] item id read by the 9 consumer warps
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 24);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 25);
  volatile int* ring_ids = reinterpret_cast<volatile int*>(bars + 26);  // [kRing]

  if (threadIdx.x == 0) {
    mbar_init(bar_kv, 1);
    for (int s = 0; s < kNQ; ++s) {
      mbar_init(&bar_q_full[s], 1);
      mbar_init(&bar_q_empty[s], 1);
    }
    mbar_init(bar_sd_full, 1);
    mbar_init(bar_sd_free, 256);
    mbar_init(bar_pds_full, 256);
    mbar_init(bar_dq_full, 1);
    mbar_init(bar_dq_free, 256);
    mbar_init(bar_done, 1);
    mbar_init(bar_pt_free, 1);
    mbar_init(bar_item, 1);
    for (int s = 0; s < kRing; ++s) {
      mbar_init(&ring_full[s], 1);
      mbar_init(&ring_empty[s], 9);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 8) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const WaitCtx wc{p.status, abort_flag, kKernelId};
  // k-th item of this CTA (consumers): wait for the producer's announcement,
  // release the ring entry; -1 = no more work or abort
  auto next_item = [&](int k, bool whole_warp) -> int {
    const int slot = k % kRing;
    const bool got = wait_bounded(wc, &ring_full[slot], (k / kRing) & 1, 18);
    const int it = got ? ring_ids[slot] : -1;
    if (whole_warp) __syncwarp();
    if (!whole_warp || lane == 0) mbar_arrive(&ring_empty[slot]);
    return it;
  };

  if (warp == 8) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&p.tm_q);
      tma_prefetch_desc(&p.tm_k);
      tma_prefetch_desc(&p.tm_v);
      tma_prefetch_desc(&p.tm_do);
      int ci = 0;   // Q/dO ring tiles issued
      int nkv = 0;  // K/V tiles issued (one per item)
      bool ok = true;
      // ring tile of item-local iteration j: query head r, query tile qi
      auto issue_ring = [&](const BwdItem& w, int j) -> bool {
        const int st = ci % kNQ;
        if (ci >= kNQ && !wait_bounded(wc, &bar_q_empty[st], ((ci / kNQ) & 1) ^ 1, 1)) return false;
        const int r = j / w.n_q;
        const int qi = w.kt + (j - r * w.n_q);
        const int h = w.hk * p.repeats + r;
        mbar_arrive_expect_tx(&bar_q_full[st], 2 * C::TILE + 2 * 512);
        tma_tile(sQ + st * C::TILE, &p.tm_q, &bar_q_full[st], qi * kBQ, h, w.b, p.sw_q);
        tma_tile(sDO + st * C::TILE, &p.tm_do, &bar_q_full[st], qi * kBQ, h, w.b, p.sw_do);
        const int64_t row0 = (int64_t(w.b) * p.Hq + h) * p.Tp + int64_t(qi) * kBQ;
        bulk_load(sLse + st * 128, p.lse2 + row0, 512, &bar_q_full[st]);
        bulk_load(sDelta + st * 128, p.delta + row0, 512, &bar_q_full[st]);
        ++ci;
        return true;
      };
      for (int k = 0; ok; ++k) {
        // take the next item from the work counter and announce it
        const int slot = k % kRing;
        if (k >= kRing && !wait_bounded(wc, &ring_empty[slot], ((k / kRing) & 1) ^ 1, 17)) break;
        int it = atomicAdd(p.sched, 1);
        if (it >= p.n_items) it = -1;
        ring_ids[slot] = it;
        mbar_arrive(&ring_full[slot]);
        if (it < 0) break;
        const BwdItem w = bwd_item(p, it);
        // after the first item: the ring runs ahead into this item while the
        // previous one finishes; K/V are replaced once its last dQ is done
        const int pre = nkv > 0 ? min(kNQ, w.n_it) : 0;
        for (int j = 0; ok && j < pre; ++j) ok = issue_ring(w, j);
        if (!ok || (nkv > 0 && !wait_bounded(wc, bar_item, (nkv - 1) & 1, 14))) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(bar_kv, 2 * C::TILE);
        tma_tile(sK, &p.tm_k, bar_kv, w.kt * kBK, w.hk, w.b, p.sw_k);
        tma_tile(sV, &p.tm_v, bar_kv, w.kt * kBK, w.hk, w.b, p.sw_v);
        ++nkv;
        for (int j = pre; ok && j < w.n_it; ++j) ok = issue_ring(w, j);
      }
      if (*abort_flag) {
        // copies already issued must land before shared memory is released
        if (nkv > 0) wait_drain(wc, bar_kv, (nkv - 1) & 1, 11);
        for (int i = (ci > kNQ ? ci - kNQ : 0); i < ci; ++i)
          wait_drain(wc, &bar_q_full[i % kNQ], (i / kNQ) & 1, 12);
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr int kBf16 = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
      constexpr uint32_t idesc_sd = make_idesc(128, kBQ, kBf16, 0, 0);  // K-major A and B
      constexpr uint32_t idesc_acc = make_idesc(128, D, kBf16, 0, 1);   // A K-major, B MN-major
      constexpr uint32_t idesc_dq = make_idesc(128, D, kBf16, 1, 1);    // A and B MN-major
      const uint32_t k_base = smem_u32(sK), v_base = smem_u32(sV);
      const uint32_t q_base = smem_u32(sQ), do_base = smem_u32(sDO);
      const uint32_t ds_base = smem_u32(sDS);
      // Descriptors are built once per operand tile and stepped by adding to
      // the start-address field (bytes / 16), which keeps the issue loop short:
      // the next MMA goes out only when this thread reaches it, and per-MMA
      // descriptor arithmetic measured ~12 cycles per N = 64 instruction.
      const uint64_t dk0 = make_sdesc(k_base, 16, C::SBO, C::LAYOUT);
      const uint64_t dv0 = make_sdesc(v_base, 16, C::SBO, C::LAYOUT);
      const uint64_t dk_mn0 = make_sdesc(k_base, C::TILE, C::SBO, C::LAYOUT);
      const uint64_t ds_k0 = make_sdesc(ds_base, 16, 1024, kSwizzle128);
      const uint64_t ds_mn0 = make_sdesc(ds_base, 128 * 128, 1024, kSwizzle128);
      constexpr uint32_t kRowStep = 16 * C::ROW_BYTES / 16;  // 16 rows of a tile, in descriptor units
      auto issue_sdp = [&](int st) {
        const uint32_t qb = q_base + st * C::TILE, dob = do_base + st * C::TILE;
        const uint64_t dq = make_sdesc(qb, 16, C::SBO, C::LAYOUT), ddo = make_sdesc(dob, 16, C::SBO, C::LAYOUT);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_ss(tmem + C::T_S, dk0 + 2 * kk, dq + 2 * kk, idesc_sd, kk > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_ss(tmem + C::T_DP, dv0 + 2 * kk, ddo + 2 * kk, idesc_sd, kk > 0 ? 1u : 0u);
        umma_commit(bar_sd_full);
      };
      // Issue order per tile i: S/dP of tile i+1 as soon as the compute warps
      // have read S/dP of tile i, then dV, dK, dQ of tile i -- so the compute
      // warps' softmax of tile i+1 overlaps the three accumulating products.
      // Counters run across items (ci: iterations, n: items).
      int ci = 0, n = 0;
      bool ok = true;
      for (int k = 0; ok; ++k, ++n) {
        const int it = next_item(k, false);
        if (it < 0) break;
        const BwdItem w = bwd_item(p, it);
        // S/dP of the item's first tile: the previous item's last S/dP was
        // read (waited in its last iteration) and this item's K/V landed
        ok = wait_bounded(wc, bar_kv, n & 1, 2) && wait_bounded(wc, &bar_q_full[ci % kNQ], (ci / kNQ) & 1, 3);
        if (ok) {
          tc_fence_after();
          issue_sdp(ci % kNQ);
        }
        for (int j = 0; ok && j < w.n_it; ++j, ++ci) {
          const int st = ci % kNQ;
          if (!wait_bounded(wc, bar_sd_free, ci & 1, 4)) {
            ok = false;
            break;
          }
          if (j + 1 < w.n_it) {
            const int c1 = ci + 1;
            if (!wait_bounded(wc, &bar_q_full[c1 % kNQ], (c1 / kNQ) & 1, 3)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_sdp(c1 % kNQ);
          }
          if (!wait_bounded(wc, bar_pds_full, ci & 1, 5)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t qb = q_base + st * C::TILE, dob = do_base + st * C::TILE;
          const uint64_t ddo_mn = make_sdesc(dob, C::TILE, C::SBO, C::LAYOUT);
          const uint64_t dq_mn = make_sdesc(qb, C::TILE, C::SBO, C::LAYOUT);
          // dV += P^T dO ; dK += dS^T Q   (K = 128 queries in steps of 16)
#pragma unroll
          for (int kk = 0; kk < kBQ / 16; ++kk) {
            const uint32_t acc = (j > 0 || kk > 0) ? 1u : 0u;
            umma_ts(tmem + C::T_DV, tmem + C::T_PT + kk * 8, ddo_mn + kRowStep * kk, idesc_acc, acc);
          }
          umma_commit(bar_pt_free);
#pragma unroll
          for (int kk = 0; kk < kBQ / 16; ++kk) {
            // dS^T K-major: 64-column atoms of 128 x 128 bytes, 32 bytes per K step inside an atom
            const uint32_t a_step = (kk >> 2) * (128 * 128 / 16) + (kk & 3) * 2;
            const uint32_t acc = (j > 0 || kk > 0) ? 1u : 0u;
            umma_ss(tmem + C::T_DK, ds_k0 + a_step, dq_mn + kRowStep * kk, idesc_acc, acc);
          }
          umma_commit(&bar_q_empty[st]);  // Q/dO of this stage are no longer read (dQ reads K and dS)
          if (ci > 0 && !wait_bounded(wc, bar_dq_free, (ci - 1) & 1, 6)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // dQ = dS K   (M = 128 queries, K = 128 keys in steps of 16)
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            umma_ss(tmem + C::T_DQ, ds_mn0 + (2048 / 16) * kk, dk_mn0 + kRowStep * kk, idesc_dq, kk > 0 ? 1u : 0u);
          umma_commit(bar_dq_full);
          if (j + 1 == w.n_it) umma_commit(bar_item);
        }
      }
      // every issued MMA completes before TMEM is released (also on abort)
      umma_commit(bar_done);
      wait_drain(wc, bar_done, 0, 13);
    }
  } else {
    // ------------------------------------------------------------ compute
    const int wg = warp >> 2;          // query-column half handled by this warpgroup
    const int r = threadIdx.x & 127;   // TMEM lane: key row (S/dP) or query row (dQ)
    const uint32_t lane_off = uint32_t((warp & 3) * 32) << 16;
    bool ok = true;
    // Drain dQ of global iteration `pit` (batch pb, query head ph, query tile
    // pq): TMEM -> swizzled fp32 staging -> TMA reduce-add into the
    // accumulator.  Returns false on abort.
    auto drain_dq = [&](int pit, int pb, int ph, int pq) -> bool {
      if (!bar_all(wait_bounded(wc, bar_dq_full, pit & 1, 9), 4, 256)) return false;
      tc_fence_after();
      constexpr int kCols = D / 2;  // dQ columns per warpgroup
      const bool leader = (threadIdx.x & 127) == 0;
      // the previous reduce of this warpgroup must have finished reading staging
      if (leader) bulk_wait_group_read0();
      named_bar_sync(1 + wg, 128);
      // TMEM -> registers -> fp32 staging (box bx = 32 columns x 128 rows,
      // 128 B rows, 128B swizzle)
      if constexpr (kCols == 32) {
        uint32_t qa[16], qb[16];
        tmem_ld16(tmem + lane_off + C::T_DQ + wg * 32, qa);
        tmem_ld16(tmem + lane_off + C::T_DQ + wg * 32 + 16, qb);
        tmem_ld_wait_regs(qa, qb);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const uint32_t* src = q < 4 ? &qa[q * 4] : &qb[(q - 4) * 4];
          const int col = wg * 32 + q * 4;
          const int ch = (col & 31) >> 2;
          *reinterpret_cast<uint4*>(sDQ + (col >> 5) * (128 * 128) + r * 128 + ((ch ^ (r & 7)) * 16)) =
              make_uint4(src[0], src[1], src[2], src[3]);
        }
      } else {
        uint32_t qa[16], qb[16];
        tmem_ld16(tmem + lane_off + C::T_DQ + wg * 16, qa);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) qb[i] = 0u;
        tmem_ld_wait_regs(qa, qb);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int col = wg * 16 + q * 4;
          const int ch = (col & 31) >> 2;
          *reinterpret_cast<uint4*>(sDQ + r * 128 + ((ch ^ (r & 7)) * 16)) =
              make_uint4(qa[q * 4], qa[q * 4 + 1], qa[q * 4 + 2], qa[q * 4 + 3]);
        }
      }
      tc_fence_before();
      mbar_arrive(bar_dq_free);
      fence_proxy_async_smem();
      const int row0 = (pb * p.Hq + ph) * p.Tp + pq * kBQ;
      if constexpr (kCols == 32) {
        named_bar_sync(1 + wg, 128);
        if (leader) {
          tma_reduce_add_2d(&p.tm_dq, sDQ + wg * (128 * 128), wg * 32, row0);
          bulk_commit_group();
        }
      } else {
        // D == 32: both halves live in box 0; one thread issues after both wrote
        named_bar_sync(3, 256);
        if (threadIdx.x == 0) {
          tma_reduce_add_2d(&p.tm_dq, sDQ, 0, row0);
          bulk_commit_group();
          bulk_wait_group_read0();
        }
        named_bar_sync(3, 256);
      }
      return true;
    };
    int ci = 0, n = 0;
    for (int k = 0; ok; ++k, ++n) {
      // one decision for both warpgroups (they meet at named barriers)
      const int item = next_item(k, true);
      if (!bar_all(item >= 0, 4, 256)) break;
      const BwdItem w = bwd_item(p, item);
      const int kt = w.kt;
      const int key = kt * kBK + r;
      int prev_h = 0, prev_q = 0;
      for (int j = 0; j < w.n_it; ++j, ++ci) {
        const int st = ci % kNQ;
        const int rr = j / w.n_q;
        const int qi = kt + (j - rr * w.n_q);
        const int h = w.hk * p.repeats + rr;
        const bool diag = (qi == kt);
        if (!bar_all(wait_bounded(wc, bar_sd_full, ci & 1, 8), 4, 256)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float* lse = sLse + st * 128;
        const float* dl = sDelta + st * 128;
        // P^T and dS^T rows for this warpgroup's 64 query columns, packed in
        // registers until the previous tile's products have released the tiles
        uint32_t pk0[16], pk1[16], dk[2][16];
        // S^T / dP^T columns of this warpgroup in four 16-column chunks; the
        // TMEM loads of chunk c+1 are in flight while chunk c is processed.
        auto process = [&](int c, const uint32_t (&sv)[16], const uint32_t (&dv)[16]) {
          const int col0 = wg * 64 + c * 16;
          const int lim = key - (qi * kBQ + col0);  // column i is masked when i < lim (key > query)
          float lv[16], dlv[16];
#pragma unroll
          for (int i = 0; i < 16; i += 4) {
            const float4 a = *reinterpret_cast<const float4*>(lse + col0 + i);
            const float4 d = *reinterpret_cast<const float4*>(dl + col0 + i);
            lv[i] = a.x; lv[i + 1] = a.y; lv[i + 2] = a.z; lv[i + 3] = a.w;
            dlv[i] = d.x; dlv[i + 1] = d.y; dlv[i + 2] = d.z; dlv[i + 3] = d.w;
          }
          const float2 sc2 = make_float2(p.scale_log2, p.scale_log2);
#pragma unroll
          for (int i = 0; i < 16; i += 2) {
            // P = exp2(s * scale * log2e - lse * log2e), dS = P (dP - delta), two lanes per instruction
            const float2 x = fma2(make_float2(__uint_as_float(sv[i]), __uint_as_float(sv[i + 1])), sc2,
                                  make_float2(lv[i], lv[i + 1]));
            float p0 = fast_exp2(x.x);
            float p1 = fast_exp2(x.y);
            if (diag) {
              if (i < lim) p0 = 0.f;
              if (i + 1 < lim) p1 = 0.f;
            }
            const float2 dd = mul2(make_float2(p0, p1), sub2(make_float2(__uint_as_float(dv[i]), __uint_as_float(dv[i + 1])),
                                                             make_float2(dlv[i], dlv[i + 1])));
            const float d0 = dd.x, d1 = dd.y;
            if (c < 2)
              pk0[(c & 1) * 8 + (i >> 1)] = pack2<T>(p0, p1);
            else
              pk1[(c & 1) * 8 + (i >> 1)] = pack2<T>(p0, p1);
            dk[c >> 1][(c & 1) * 8 + (i >> 1)] = pack2<T>(d0, d1);
          }
        };
        {
          const uint32_t ts = tmem + lane_off + C::T_S + wg * 64;
          const uint32_t td = tmem + lane_off + C::T_DP + wg * 64;
          uint32_t sa[16], da[16], sb[16], db[16];
          tmem_ld16(ts, sa);
          tmem_ld16(td, da);
          tmem_ld_wait_regs(sa, da);
          tmem_ld16(ts + 16, sb);
          tmem_ld16(td + 16, db);
          process(0, sa, da);
          tmem_ld_wait_regs(sb, db);
          tmem_ld16(ts + 32, sa);
          tmem_ld16(td + 32, da);
          process(1, sb, db);
          // P^T -> TMEM as soon as dV of the previous tile has released it
          // (an item's first tile: the previous item's last dV is complete)
          if (j > 0 && !bar_all(wait_bounded(wc, bar_pt_free, (ci - 1) & 1, 7), 4, 256)) {
            ok = false;
          } else {
            tc_fence_after();
            tmem_st16(tmem + lane_off + C::T_PT + wg * 32, pk0);
          }
          tmem_ld_wait_regs(sa, da);
          tmem_ld16(ts + 48, sb);
          tmem_ld16(td + 48, db);
          process(2, sa, da);
          tmem_ld_wait_regs(sb, db);
          process(3, sb, db);
          if (ok) tmem_st16(tmem + lane_off + C::T_PT + wg * 32 + 16, pk1);
        }
        if (!ok) break;
        tc_fence_before();
        mbar_arrive(bar_sd_free);
        // dV/dK/dQ of the previous tile are complete once its dQ is: then the
        // P/dS tiles are free and its dQ can be drained
        if (j > 0 && !drain_dq(ci - 1, w.b, prev_h, prev_q)) {
          ok = false;
          break;
        }
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int col0 = wg * 64 + c * 32;
          uint8_t* db = sDS + (col0 >> 6) * (128 * 128) + r * 128;
          const int ch0 = (col0 & 63) >> 3;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int off = ((ch0 + q) ^ (r & 7)) * 16;
            *reinterpret_cast<uint4*>(db + off) = make_uint4(dk[c][q * 4], dk[c][q * 4 + 1], dk[c][q * 4 + 2], dk[c][q * 4 + 3]);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        fence_proxy_async_smem();
        mbar_arrive(bar_pds_full);
        prev_h = h;
        prev_q = qi;
      }
      if (!ok || !drain_dq(ci - 1, w.b, prev_h, prev_q)) {
        ok = false;
        break;
      }
      // final: dV and dK (scaled) for this key tile, once the item's MMAs are done.
      // They are read before this warpgroup announces the next item's first
      // P/dS tile, so the next item's first dV/dK (which overwrite them) wait.
      if (!bar_all(wait_bounded(wc, bar_item, n & 1, 10), 4, 256)) {
        ok = false;
        break;
      }
      {
        tc_fence_after();
        constexpr int kCols = D / 2;
        uint32_t vv[kCols], kv[kCols];
        if constexpr (kCols == 32) {
          tmem_ld32(tmem + lane_off + C::T_DV + wg * 32, *reinterpret_cast<uint32_t(*)[32]>(vv));
          tmem_ld32(tmem + lane_off + C::T_DK + wg * 32, *reinterpret_cast<uint32_t(*)[32]>(kv));
        } else {
          tmem_ld16(tmem + lane_off + C::T_DV + wg * 16, *reinterpret_cast<uint32_t(*)[16]>(vv));
          tmem_ld16(tmem + lane_off + C::T_DK + wg * 16, *reinterpret_cast<uint32_t(*)[16]>(kv));
        }
        tmem_ld_wait();
        tc_fence_before();
        if (key < p.T) {
          T* dvrow = static_cast<T*>(p.dv) + int64_t(w.b) * p.dvs[0] + int64_t(w.hk) * p.dvs[1] +
                     int64_t(key) * p.dvs[2] + wg * kCols;
          T* dkrow = static_cast<T*>(p.dk) + int64_t(w.b) * p.dks[0] + int64_t(w.hk) * p.dks[1] +
                     int64_t(key) * p.dks[2] + wg * kCols;
#pragma unroll
          for (int q = 0; q < kCols / 8; ++q) {
            uint4 a, c;
            a.x = pack2<T>(__uint_as_float(vv[q * 8 + 0]), __uint_as_float(vv[q * 8 + 1]));
            a.y = pack2<T>(__uint_as_float(vv[q * 8 + 2]), __uint_as_float(vv[q * 8 + 3]));
            a.z = pack2<T>(__uint_as_float(vv[q * 8 + 4]), __uint_as_float(vv[q * 8 + 5]));
            a.w = pack2<T>(__uint_as_float(vv[q * 8 + 6]), __uint_as_float(vv[q * 8 + 7]));
            float g[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) g[i] = __uint_as_float(kv[q * 8 + i]) * p.scale;
            if (p.rope_cos != nullptr) rope_back8<T>(g, p.rope_cos, p.rope_sin, p.rope_ld, key, (wg * kCols + q * 8) / 2);
            c.x = pack2<T>(g[0], g[1]);
            c.y = pack2<T>(g[2], g[3]);
            c.z = pack2<T>(g[4], g[5]);
            c.w = pack2<T>(g[6], g[7]);
            *reinterpret_cast<uint4*>(dvrow + q * 8) = a;
            *reinterpret_cast<uint4*>(dkrow + q * 8) = c;
          }
        }
      }
    }
    // outstanding dQ reductions must finish before the CTA's shared memory goes away
    if ((threadIdx.x & 127) == 0) bulk_wait_group0();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// preprocess: delta = rowsum(O * dO), lse2 = -lse * log2(e) (-inf past T: P = 0
// there), stored negated so the probability is one fma + ex2; zeroes the fp32
// dQ accumulator rows and the main kernel's work counter
// 8 (D=64) or 4 (D=32) lanes per row, 16-byte loads.
// ---------------------------------------------------------------------------
template <typename T, int D>
__global__ void __launch_bounds__(256) attn_bwd_pre(const T* __restrict__ o, const T* __restrict__ dout,
                                                    const float* __restrict__ lse, float* __restrict__ delta,
                                                    float* __restrict__ lse2, float* __restrict__ dq_acc,
                                                    int64_t os0, int64_t os1, int64_t os2,
                                                    int64_t ds0, int64_t ds1, int64_t ds2, int Hq, int seq, int Tp,
                                                    int64_t rows, int* __restrict__ sched) {
  constexpr int LPR = D / 8;  // lanes per row
  const int64_t gid = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (gid == 0) *sched = 0;  // the main kernel's work counter
  const int64_t row = gid / LPR;
  const int sub = (int)(gid % LPR);
  const bool valid_row = row < rows;
  int64_t bh = valid_row ? row / Tp : 0;
  const int t = valid_row ? (int)(row - bh * Tp) : 0;
  const int b = (int)(bh / Hq), h = (int)(bh - int64_t(b) * Hq);
  float acc = 0.f;
  if (valid_row && t < seq) {
    float a[8], c[8];
    load_vec<T, 8>(o + b * os0 + h * os1 + int64_t(t) * os2 + sub * 8, a);
    load_vec<T, 8>(dout + b * ds0 + h * ds1 + int64_t(t) * ds2 + sub * 8, c);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc = fmaf(a[i], c[i], acc);
  }
#pragma unroll
  for (int off = LPR / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (valid_row) {  // the fp32 dQ accumulator starts at zero
    float4* z = reinterpret_cast<float4*>(dq_acc + row * D + sub * 8);
    z[0] = make_float4(0.f, 0.f, 0.f, 0.f);
    z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (valid_row && sub == 0) {
    delta[row] = acc;
    lse2[row] = (t < seq) ? lse[bh * seq + t] * -1.4426950408889634f : -INFINITY;
  }
}

// postprocess: dq[b,h,t,:] = scale * dq_acc[row, :]
// (with RoPE tables: rotated back by -theta(t) before rounding)
template <typename T, int D>
__global__ void __launch_bounds__(256) attn_bwd_post(const float* __restrict__ acc, T* __restrict__ dq,
                                                     int64_t s0, int64_t s1, int64_t s2, int Hq, int seq, int Tp,
                                                     float scale, int64_t rows, const void* rope_cos,
                                                     const void* rope_sin, int64_t rope_ld) {
  constexpr int LPR = D / 8;
  const int64_t gid = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t row = gid / LPR;
  const int sub = (int)(gid % LPR);
  if (row >= rows) return;
  const int64_t bh = row / Tp;
  const int t = (int)(row - bh * Tp);
  if (t >= seq) return;
  const int b = (int)(bh / Hq), h = (int)(bh - int64_t(b) * Hq);
  const float4* src = reinterpret_cast<const float4*>(acc + row * D + sub * 8);
  const float4 x = src[0], y = src[1];
  float v[8] = {x.x * scale, x.y * scale, x.z * scale, x.w * scale,
                y.x * scale, y.y * scale, y.z * scale, y.w * scale};
  if (rope_cos != nullptr) rope_back8<T>(v, rope_cos, rope_sin, rope_ld, t, sub * 4);
  store_vec<T, 8>(dq + b * s0 + h * s1 + int64_t(t) * s2 + sub * 8, v);
}

struct Workspace {
  float* delta;
  float* lse2;
  float* dq_acc;
  int* sched;
  int64_t bytes;
};

Workspace carve(void* base, int64_t B, int64_t Hq, int64_t T, int64_t D) {
  const int64_t Tp = (T + 127) / 128 * 128;
  const int64_t rows = B * Hq * Tp;
  auto up = [](int64_t x) { return (x + 255) / 256 * 256; };
  Workspace w;
  char* p = static_cast<char*>(base);
  const int64_t a = up(rows * 4), c = up(rows * D * 4);
  w.delta = reinterpret_cast<float*>(p);
  w.lse2 = reinterpret_cast<float*>(p + a);
  w.dq_acc = reinterpret_cast<float*>(p + 2 * a);
  w.sched = reinterpret_cast<int*>(p + 2 * a + c);
  w.bytes = 2 * a + c + 256;
  return w;
}

template <typename T, int D>
int run_bwd(BwdParams& prm, const void* o, const void* dout, const float* lse, void* dq, const int64_t* os,
            const int64_t* dos, const int64_t* dqs, Workspace& ws, int B, cudaStream_t stream) {
  using C = BwdCfg<D>;
  const int64_t rows = int64_t(B) * prm.Hq * prm.Tp;
  {
    const int64_t threads = rows * (D / 8);
    attn_bwd_pre<T, D><<<(unsigned)((threads + 255) / 256), 256, 0, stream>>>(
        static_cast<const T*>(o), static_cast<const T*>(dout), lse, ws.delta, ws.lse2, ws.dq_acc, os[0], os[1], os[2], dos[0],
        dos[1], dos[2], prm.Hq, prm.T, prm.Tp, rows, ws.sched);
    int st = check_launch("attention_bwd_pre");
    if (st != MT_OK) return st;
  }
  {
    auto kern = attn_bwd_kernel<T, D>;
    int st = set_smem_limit((const void*)kern, C::SMEM);
    if (st != MT_OK) return st;
    // group size: about 32 MB of Q + dO (16-bit) and fp32 dQ rows per group
    const int64_t head_bytes = int64_t(prm.repeats) * prm.Tp * D * 8;
    const int64_t g = (int64_t(32) << 20) / (head_bytes > 0 ? head_bytes : 1);
    prm.n_heads = B * prm.Hkv;
    prm.group = (int)(g < 1 ? 1 : (g > prm.n_heads ? prm.n_heads : g));
    const int64_t items = int64_t(prm.n_heads) * prm.n_tiles;
    if (items > 0x7fffffff) return MT_ERR_INVALID_ARGUMENT;
    prm.n_items = (int)items;
    // persistent: one CTA per SM (the kernel's shared memory and TMEM allow one)
    const int blocks = prm.n_items < get_sm_count() ? prm.n_items : get_sm_count();
    record_timing_event(0, stream);
    kern<<<(unsigned)blocks, kThreads, C::SMEM, stream>>>(prm);
    record_timing_event(1, stream);
    st = check_launch("attention_bwd");
    if (st != MT_OK) return st;
  }
  {
    const int64_t threads = rows * (D / 8);
    attn_bwd_post<T, D><<<(unsigned)((threads + 255) / 256), 256, 0, stream>>>(
        ws.dq_acc, static_cast<T*>(dq), dqs[0], dqs[1], dqs[2], prm.Hq, prm.T, prm.Tp, prm.scale, rows,
        prm.rope_cos, prm.rope_sin, prm.rope_ld);
    return check_launch("attention_bwd_post");
  }
}

}  // namespace
}  // namespace mt

using namespace mt;

extern "C" int64_t mt_attention_bwd_workspace_bytes(int64_t B, int64_t Hq, int64_t T, int64_t D) {
  if (B <= 0 || Hq <= 0 || T <= 0 || D <= 0) return 0;
  return carve(nullptr, B, Hq, T, D).bytes;
}

static int attention_bwd_impl(const void* q, const void* k, const void* v, const void* o, const float* lse,
                              const void* dout, void* dq, void* dk, void* dv, int dtype, int64_t B, int64_t Hq,
                              int64_t Hkv, int64_t T, int64_t D, const int64_t* qs, const int64_t* ks,
                              const int64_t* vs, const int64_t* os, const int64_t* dos, const int64_t* dqs,
                              const int64_t* dks, const int64_t* dvs, float scale, const void* rope_cos,
                              const void* rope_sin, int64_t rope_ld, void* workspace, int64_t workspace_bytes,
                              uint32_t* status, void* stream) {
  if (dtype != MT_BF16 && dtype != MT_F16) return MT_ERR_UNSUPPORTED_DTYPE;
  if (B < 0 || Hq <= 0 || Hkv <= 0 || T < 0 || (Hq % Hkv) != 0) return MT_ERR_INVALID_ARGUMENT;
  if (D != 64 && D != 32) return MT_ERR_INVALID_ARGUMENT;
  if (B == 0 || T == 0) return MT_OK;
  if (lse == nullptr || status == nullptr) return MT_ERR_INVALID_ARGUMENT;
  const int64_t Tp = (T + 127) / 128 * 128;
  if (B * Hq * Tp > 0x7fffffffLL || B * Hkv > 0x7fffffffLL) return MT_ERR_INVALID_ARGUMENT;
  int st = MT_OK;
  const void* ptrs[9] = {q, k, v, o, dout, dq, dk, dv, nullptr};
  const int64_t* strides[8] = {qs, ks, vs, os, dos, dqs, dks, dvs};
  for (int i = 0; i < 8; ++i)
    if ((st = check_attn_layout(ptrs[i], strides[i], true)) != MT_OK) return st;
  if (workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return MT_ERR_WORKSPACE;
  Workspace ws = carve(workspace, B, Hq, T, D);
  if (workspace_bytes < ws.bytes) return MT_ERR_WORKSPACE;
  if ((st = bind_device_of(q)) != MT_OK) return st;
  if ((st = check_arch()) != MT_OK) return st;

  BwdParams prm;
  // coordinate orders: q/k/v follow the forward's choice; dO gets its own
  int swq = (Hq == 1 || T == 1) ? 0 : -1;
  if ((st = make_bhtd_map(&prm.tm_q, q, dtype, B, Hq, T, D, qs, kBQ, &swq)) != MT_OK) return st;
  int swk = (Hkv == 1 || T == 1) ? 0 : -1, swv = swk, swdo = (Hq == 1 || T == 1) ? 0 : -1;
  if ((st = make_bhtd_map(&prm.tm_k, k, dtype, B, Hkv, T, D, ks, kBK, &swk)) != MT_OK) return st;
  if ((st = make_bhtd_map(&prm.tm_v, v, dtype, B, Hkv, T, D, vs, kBK, &swv)) != MT_OK) return st;
  if ((st = make_bhtd_map(&prm.tm_do, dout, dtype, B, Hq, T, D, dos, kBQ, &swdo)) != MT_OK) return st;
  {
    // fp32 dQ accumulator as a 2-D tensor [B*Hq*Tp rows, D] with 32-column boxes
    uint64_t dims[2] = {(uint64_t)D, (uint64_t)(B * Hq * Tp)};
    uint64_t strides_b[1] = {(uint64_t)(D * 4)};
    uint32_t box[2] = {32, 128};
    if ((st = encode_tensor_map(&prm.tm_dq, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, ws.dq_acc, dims, strides_b, box,
                                CU_TENSOR_MAP_SWIZZLE_128B)) != MT_OK)
      return st;
  }
  prm.sw_q = swq;
  prm.sw_k = swk;
  prm.sw_v = swv;
  prm.sw_do = swdo;
  prm.lse2 = ws.lse2;
  prm.delta = ws.delta;
  prm.sched = ws.sched;
  prm.dk = dk;
  prm.dv = dv;
  prm.rope_cos = rope_cos;
  prm.rope_sin = rope_sin;
  prm.rope_ld = rope_ld;
  for (int i = 0; i < 4; ++i) {
    prm.dks[i] = dks[i];
    prm.dvs[i] = dvs[i];
  }
  prm.T = (int)T;
  prm.Tp = (int)Tp;
  prm.Hq = (int)Hq;
  prm.Hkv = (int)Hkv;
  prm.repeats = (int)(Hq / Hkv);
  prm.n_tiles = (int)(Tp / 128);
  prm.scale = scale;
  prm.scale_log2 = scale * 1.4426950408889634f;
  prm.status = status;
  if (prm.n_tiles > 65535) return MT_ERR_INVALID_ARGUMENT;
  auto s = static_cast<cudaStream_t>(stream);
  const bool bf = dtype == MT_BF16;
  const int b = (int)B;
  if (D == 64)
    return bf ? run_bwd<__nv_bfloat16, 64>(prm, o, dout, lse, dq, os, dos, dqs, ws, b, s)
              : run_bwd<__half, 64>(prm, o, dout, lse, dq, os, dos, dqs, ws, b, s);
  return bf ? run_bwd<__nv_bfloat16, 32>(prm, o, dout, lse, dq, os, dos, dqs, ws, b, s)
            : run_bwd<__half, 32>(prm, o, dout, lse, dq, os, dos, dqs, ws, b, s);
}

extern "C" int mt_attention_bwd(const void* q, const void* k, const void* v, const void* o, const float* lse,
                                const void* dout, void* dq, void* dk, void* dv, int dtype, int64_t B, int64_t Hq,
                                int64_t Hkv, int64_t T, int64_t D, const int64_t* qs, const int64_t* ks,
                                const int64_t* vs, const int64_t* os, const int64_t* dos, const int64_t* dqs,
                                const int64_t* dks, const int64_t* dvs, float scale, void* workspace,
                                int64_t workspace_bytes, uint32_t* status, void* stream) {
  return attention_bwd_impl(q, k, v, o, lse, dout, dq, dk, dv, dtype, B, Hq, Hkv, T, D, qs, ks, vs, os, dos, dqs, dks,
                            dvs, scale, nullptr, nullptr, 0, workspace, workspace_bytes, status, stream);
}

extern "C" int mt_attention_rope_bwd(const void* q, const void* k, const void* v, const void* o, const float* lse,
                                     const void* dout, void* dq, void* dk, void* dv, int dtype, int64_t B,
                                     int64_t Hq, int64_t Hkv, int64_t T, int64_t D, const int64_t* qs,
                                     const int64_t* ks, const int64_t* vs, const int64_t* os, const int64_t* dos,
                                     const int64_t* dqs, const int64_t* dks, const int64_t* dvs, float scale,
                                     const void* rope_cos, const void* rope_sin, int64_t rope_ld, void* workspace,
                                     int64_t workspace_bytes, uint32_t* status, void* stream) {
  if (rope_cos == nullptr || rope_sin == nullptr || rope_ld < D / 2) return MT_ERR_INVALID_ARGUMENT;
  // 8-byte table reads: 4 pairs at a time
  if ((reinterpret_cast<uintptr_t>(rope_cos) & 7u) || (reinterpret_cast<uintptr_t>(rope_sin) & 7u) ||
      (rope_ld % 4) != 0)
    return MT_ERR_UNSUPPORTED_LAYOUT;
  return attention_bwd_impl(q, k, v, o, lse, dout, dq, dk, dv, dtype, B, Hq, Hkv, T, D, qs, ks, vs, os, dos, dqs, dks,
                            dvs, scale, rope_cos, rope_sin, rope_ld, workspace, workspace_bytes, status, stream);
}
