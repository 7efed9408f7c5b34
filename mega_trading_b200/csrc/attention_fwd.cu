// Causal grouped-query flash attention, forward, for sm_100a.
//
// Reference semantics (duoan/mega-trading):
//   src/mega_trading/kernels/triton_attention.py:12-24 (validation), :27-78
//   (forward: O and fp32 logsumexp saved for backward, scale = 1/sqrt(D)),
//   :260-358 / :361-478 (online-softmax kernels).  Torch oracle:
//   F.scaled_dot_product_attention(is_causal=True, enable_gqa=True)
//   (model.py:228-235).
//
// B200 design
//   * Work item = two consecutive 128-row query tiles ("slots") of one
//     (batch, query head); both slots share one K/V tile stream (3 stages).
//     Persistent: one CTA per SM (128 KB smem, all 512 TMEM columns) takes
//     items from a global work counter (zeroed in the caller's workspace
//     before the launch; the producer warp fetches each item and passes it
//     to the MMA and softmax warps through a shared-memory ring), so the next
//     item's Q load and first S = Q K^T overlap this item's last softmax and
//     epilogue, items of unequal causal length balance across SMs, and
//     barrier setup and TMEM allocation happen once per SM.
//   * Warp roles: warps 0-3 / 4-7 = softmax of slot 0 / 1 (thread i owns TMEM
//     lane = query row i of its slot), warp 8 = TMA producer (+ TMEM
//     allocation), warp 9 = tcgen05.mma issuer.
//   * Per slot s: S = Q K^T (M=128, N=128, K=D) accumulates in TMEM columns
//     [256s, 256s+128); O += P V (M=128, N=D, K=128) in [256s+128, 256s+128+D);
//     P lives in [256s+192, 256s+256).
//   * Q/K/V tiles arrive by TMA (one copy per CTA) in the 128B (D=64) or 64B (D=32)
//     swizzle that the UMMA shared-memory descriptors expect; V is consumed
//     MN-major so it needs no transpose.  K/V are double-buffered.
//   * P is rounded to the input dtype (as the reference does before its PV
//     dot, triton_attention.py:340) and stored into TMEM next to S and O; the
//     P V product reads it from TMEM (tcgen05.mma with a TMEM A operand), so
//     only V is read from shared memory (shared-memory bandwidth, not the
//     tensor core, limits an all-shared-memory P V at N = D = 64).
//   * Causal: key tiles 0..qtile only; the diagonal tile is masked in
//     registers.  Items are ordered heaviest query tile first.
//   * Every mbarrier wait is bounded (status word + early exit, no trap).
#include <cmath>
#include <type_traits>

#include "common.cuh"

namespace mt {
namespace {

constexpr int kBM = 128;  // query rows per slot
constexpr int kBN = 128;  // keys per tile
constexpr int kSlots = 2;  // query tiles per CTA (consecutive tiles of one head)
constexpr int kThreads = 352;  // 8 softmax warps, 1 TMA warp, 2 MMA warps
constexpr int kRing = 4;       // work items announced ahead by the producer warp
// Of every 8 pairs of scores, kPolyPairs take the polynomial exp2 on the FMA
// pipe and the rest the MUFU ex2 (16 per clock per SM), the forward's
// bottleneck at D=64: measured best at 2 (654 vs 646 at 1, 628 at 3 TFLOP/s
// at T=4096; 676 vs 621 / 628 at B=128, Hq 12, T=2048, and best at T=1024).
constexpr int kPolyPairs = 2;
constexpr uint32_t kKernelId = 1;

template <int D>
struct FwdCfg {
  static constexpr int ROW_BYTES = D * 2;
  static constexpr uint32_t LAYOUT = (D == 64) ? kSwizzle128 : kSwizzle64;
  static constexpr int SBO = 8 * ROW_BYTES;  // bytes between 8-row core groups
  static constexpr int TILE = kBM * ROW_BYTES;
  static constexpr int NST = 3;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + kSlots * TILE;
  static constexpr int OFF_V = OFF_K + NST * TILE;
  static constexpr int OFF_BAR = OFF_V + NST * TILE;
  static constexpr int SMEM = OFF_BAR + 512;
  // TMEM per slot s (256 columns): S fp32 [0,128), O fp32 [128,128+D),
  // P (bf16/fp16 pairs, the A operand of P V) [192,256)
  static constexpr int TMEM_COLS = 512;
  static constexpr int T_O = 128, T_P = 192;
};

struct FwdParams {
  CUtensorMap tm_q, tm_k, tm_v;
  void* o;
  float* lse;
  int64_t os[4];
  int T, Hq, Hkv, repeats, n_qtiles, n_pairs, n_items;
  int* sched;  // work counter (next item), zero at launch
  int ht_swapped;  // tensor-map coordinate order (D, H, T, B) instead of (D, T, H, B)
  float scale_log2;
  uint32_t* status;
};

__device__ __forceinline__ void tma_tile(void* dst, const CUtensorMap* map, uint64_t* bar, int t0, int h, int b,
                                         int swapped) {
  if (swapped)
    tma_load_4d(dst, map, bar, 0, h, t0, b);
  else
    tma_load_4d(dst, map, bar, 0, t0, h, b);
}

// Item order: one (batch, kv head) after another; inside it the query-tile
// pairs go heaviest first, and the `repeats` query heads of one pair are
// adjacent.  The items resident at one time then share a few kv heads, so
// their K/V tiles come from DRAM about once.
struct FwdItem {
  int b, hk, h, pair;
  int nkv0, nkv1, n_kv;  // key tiles seen by slot 0, slot 1 (0: no slot 1) and the item
};

__device__ __forceinline__ FwdItem fwd_item(const FwdParams& p, int it) {
  FwdItem w;
  const int per_kv = p.n_pairs * p.repeats;
  const int bk = it / per_kv;
  const int rem = it - bk * per_kv;
  const int pi = rem / p.repeats;
  w.b = bk / p.Hkv;
  w.hk = bk - w.b * p.Hkv;
  w.h = w.hk * p.repeats + (rem - pi * p.repeats);
  w.pair = p.n_pairs - 1 - pi;  // heaviest pair first
  // slot s handles query tile 2*pair + s; it sees key tiles 0..(2*pair + s)
  const bool active1 = (2 * w.pair + 1) < p.n_qtiles;
  w.nkv0 = 2 * w.pair + 1;
  w.nkv1 = active1 ? 2 * w.pair + 2 : 0;
  w.n_kv = active1 ? w.nkv1 : w.nkv0;
  return w;
}

template <typename T, int D>
__global__ void __launch_bounds__(kThreads, 1) attn_fwd_kernel(const __grid_constant__ FwdParams p) {
  using C = FwdCfg<D>;
  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = warp_id();
  const int lane = lane_id();
  if ((smem_u32(smem) & 1023u) != 0) {  // swizzled tiles need 1 KB alignment
    if (threadIdx.x == 0) atomicCAS(p.status, 0u, (kKernelId << 16) | 0xFFFFu);
    return;
  }
  uint8_t* sQ = smem + C::OFF_Q;
  uint8_t* sK = smem + C::OFF_K;
  uint8_t* sV = smem + C::OFF_V;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* bar_q = bars + 0;                    // [kSlots]
  uint64_t* bar_k_full = bars + 2;               // [NST]
  uint64_t* bar_v_full = bar_k_full + C::NST;    // [NST]
  uint64_t* bar_kv_empty = bar_v_full + C::NST;  // [NST]
  uint64_t* bar_s_full = bar_kv_empty + C::NST;  // [kSlots]
  uint64_t* bar_s_free = bar_s_full + kSlots;    // [kSlots]
  uint64_t* bar_p_full = bar_s_free + kSlots;    // [kSlots]
  uint64_t* bar_o_done = bar_p_full + kSlots;    // [kSlots] (+kSlots: final MMA drains)
  uint64_t* bar_q_free = bar_o_done + 2 * kSlots;  // [kSlots]: last S of an item read its Q tile
  uint64_t* ring_full = bar_q_free + kSlots;       // [kRing] item id published
  uint64_t* ring_empty = ring_full + kRing;        // [kRing] item id read by the 10 consumer warps
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 40);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 41);
  volatile int* ring_ids = reinterpret_cast<volatile int*>(bars + 42);  // [kRing]

  // Every K/V stage is released by two arrivals, one per slot: a commit after
  // the slot's P V read it, or a plain arrival from a slot that does not read
  // that tile (slot 0 on its item's last tile, slot 1 of an item without a
  // second query tile) once the tile's load has been issued.
  if (threadIdx.x == 0) {
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&bar_q[s], 1);
      mbar_init(&bar_q_free[s], 1);
      mbar_init(&bar_s_full[s], 1);
      mbar_init(&bar_s_free[s], 128);
      mbar_init(&bar_p_full[s], 128);
      mbar_init(&bar_o_done[s], 1);
    }
    mbar_init(bar_o_done + kSlots, 1);      // final MMA drain, slot 0
    mbar_init(bar_o_done + kSlots + 1, 1);  // final MMA drain, slot 1
    for (int s = 0; s < C::NST; ++s) {
      mbar_init(&bar_k_full[s], 1);
      mbar_init(&bar_v_full[s], 1);
      mbar_init(&bar_kv_empty[s], kSlots);
    }
    for (int s = 0; s < kRing; ++s) {
      mbar_init(&ring_full[s], 1);
      mbar_init(&ring_empty[s], 10);
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
      int g = 0;             // K/V tiles issued by this CTA
      int nq[kSlots] = {0, 0};  // Q tiles issued per slot
      bool ok = true;
      for (int k = 0; ok; ++k) {
        // take the next item from the work counter and announce it
        const int slot = k % kRing;
        if (k >= kRing && !wait_bounded(wc, &ring_empty[slot], ((k / kRing) & 1) ^ 1, 17)) break;
        int it = atomicAdd(p.sched, 1);
        if (it >= p.n_items) it = -1;
        ring_ids[slot] = it;
        mbar_arrive(&ring_full[slot]);
        if (it < 0) break;
        const FwdItem w = fwd_item(p, it);
        for (int s = 0; s < (w.nkv1 > 0 ? 2 : 1); ++s) {
          if (nq[s] > 0 && !wait_bounded(wc, &bar_q_free[s], (nq[s] - 1) & 1, 14)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&bar_q[s], C::TILE);
          tma_tile(sQ + s * C::TILE, &p.tm_q, &bar_q[s], (2 * w.pair + s) * kBM, w.h, w.b, p.ht_swapped);
          ++nq[s];
        }
        for (int j = 0; ok && j < w.n_kv; ++j, ++g) {
          const int st = g % C::NST;
          if (g >= C::NST && !wait_bounded(wc, &bar_kv_empty[st], ((g / C::NST) & 1) ^ 1, 1)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&bar_k_full[st], C::TILE);
          tma_tile(sK + st * C::TILE, &p.tm_k, &bar_k_full[st], j * kBN, w.hk, w.b, p.ht_swapped);
          mbar_arrive_expect_tx(&bar_v_full[st], C::TILE);
          tma_tile(sV + st * C::TILE, &p.tm_v, &bar_v_full[st], j * kBN, w.hk, w.b, p.ht_swapped);
        }
      }
      if (*abort_flag) {
        // copies already issued must land before shared memory is released
        for (int s = 0; s < kSlots; ++s)
          if (nq[s] > 0) wait_drain(wc, &bar_q[s], (nq[s] - 1) & 1, 11);
        for (int j = (g > C::NST ? g - C::NST : 0); j < g; ++j) {
          wait_drain(wc, &bar_k_full[j % C::NST], (j / C::NST) & 1, 12);
          wait_drain(wc, &bar_v_full[j % C::NST], (j / C::NST) & 1, 12);
        }
      }
    }
  } else if (warp >= 9) {
    // ------------------------------------------------------------ MMA issuers
    if (lane == 0) {
      constexpr int kBf16 = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
      constexpr uint32_t idesc_s = make_idesc(kBM, kBN, kBf16, 0, 0);
      constexpr uint32_t idesc_o = make_idesc(kBM, D, kBf16, 0, 1);
      const uint32_t q_base = smem_u32(sQ);
      const uint32_t k_base = smem_u32(sK);
      const uint32_t v_base = smem_u32(sV);
      // Descriptors built once per tile and stepped in the start-address field
      // (bytes / 16): the next MMA goes out only when this thread reaches it,
      // so the issue loop carries no per-MMA descriptor arithmetic.
      auto issue_s = [&](int slot, int st) {
        const uint64_t ad = make_sdesc(q_base + slot * C::TILE, 16, C::SBO, C::LAYOUT);
        const uint64_t bd = make_sdesc(k_base + st * C::TILE, 16, C::SBO, C::LAYOUT);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) umma_ss(tmem + slot * 256, ad + 2 * kk, bd + 2 * kk, idesc_s, kk > 0 ? 1u : 0u);
      };
      auto issue_pv = [&](int slot, int st, bool acc_first) {
        // A = P from TMEM (16 keys = 8 packed columns per step), B = V (MN-major)
        const uint64_t bd = make_sdesc(v_base + st * C::TILE, C::TILE, C::SBO, C::LAYOUT);
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk)
          umma_ts(tmem + slot * 256 + C::T_O, tmem + slot * 256 + C::T_P + kk * 8, bd + kk * C::ROW_BYTES, idesc_o,
                  (acc_first || kk > 0) ? 1u : 0u);
      };
      // One issuing thread per slot: each slot's S(j+1) goes out as soon as
      // that slot has read S(j), and its P V(j) as soon as it has written
      // P(j), whatever the other slot is doing.
      const int slot = warp - 9;
      int g = 0;   // K/V tiles of the CTA's items so far
      int cs = 0;  // S products issued
      int cp = 0;  // P V products issued
      int nq = 0;  // Q tiles used
      bool ok = true;
      for (int k = 0; ok; ++k) {
        const int it = next_item(k, false);
        if (it < 0) break;
        const FwdItem w = fwd_item(p, it);
        const int nkv = slot ? w.nkv1 : w.nkv0;
        if (nkv > 0) {
          ok = wait_bounded(wc, &bar_q[slot], nq & 1, 2) &&
               wait_bounded(wc, &bar_k_full[g % C::NST], (g / C::NST) & 1, 3) &&
               (cs == 0 || wait_bounded(wc, &bar_s_free[slot], (cs - 1) & 1, 5));
          if (ok) {
            tc_fence_after();
            issue_s(slot, g % C::NST);
            umma_commit(&bar_s_full[slot]);
            ++cs;
            if (nkv == 1) umma_commit(&bar_q_free[slot]);
          }
          for (int j = 0; ok && j < nkv; ++j) {
            const int gj = g + j;
            const int st = gj % C::NST;
            if (j + 1 < nkv) {
              const int g1 = gj + 1;
              if (!wait_bounded(wc, &bar_k_full[g1 % C::NST], (g1 / C::NST) & 1, 4) ||
                  !wait_bounded(wc, &bar_s_free[slot], (cs - 1) & 1, 5)) {
                ok = false;
                break;
              }
              tc_fence_after();
              issue_s(slot, g1 % C::NST);
              umma_commit(&bar_s_full[slot]);
              ++cs;
              if (j + 2 == nkv) umma_commit(&bar_q_free[slot]);  // the item's last S has been issued
            }
            if (!wait_bounded(wc, &bar_v_full[st], (gj / C::NST) & 1, 7) ||
                !wait_bounded(wc, &bar_p_full[slot], cp & 1, 6)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_pv(slot, st, j > 0);
            umma_commit(&bar_o_done[slot]);
            umma_commit(&bar_kv_empty[st]);  // this slot's release of the stage
            ++cp;
          }
          ++nq;
        }
        // tiles of the item this slot does not read: release them once loaded
        for (int j = nkv; ok && j < w.n_kv; ++j) {
          const int gj = g + j;
          if (!wait_bounded(wc, &bar_v_full[gj % C::NST], (gj / C::NST) & 1, 15)) {
            ok = false;
            break;
          }
          mbar_arrive(&bar_kv_empty[gj % C::NST]);
        }
        g += w.n_kv;
      }
      // every issued MMA completes before TMEM is released (also on abort)
      uint64_t* bar_fin = bar_o_done + kSlots + slot;
      umma_commit(bar_fin);
      wait_drain(wc, bar_fin, 0, 13);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int slot = warp >> 2;
    const int r = threadIdx.x & 127;  // query row within the tile == TMEM lane
    const uint32_t lane_off = uint32_t((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + slot * 256 + lane_off;
    const uint32_t tO = tS + C::T_O;
    const uint32_t tP = tS + C::T_P;
    int cs = 0;  // S tiles read
    int cp = 0;  // P tiles written
    bool ok = true;
    for (int k = 0; ok; ++k) {
      const int it = next_item(k, true);
      if (it < 0) break;
      const FwdItem w = fwd_item(p, it);
      const int nkv = slot ? w.nkv1 : w.nkv0;
      if (nkv == 0) continue;
      const int qt = 2 * w.pair + slot;
      const int qrow = qt * kBM + r;
      float m = -INFINITY;
      float l = 0.f;
      for (int j = 0; j < nkv; ++j) {
        if (!__all_sync(0xffffffffu, wait_bounded(wc, &bar_s_full[slot], cs & 1, 8))) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sv[kBN];
#pragma unroll
        for (int c = 0; c < kBN / 32; ++c) {
          uint32_t (&chunk)[32] = *reinterpret_cast<uint32_t(*)[32]>(&sv[c * 32]);
          tmem_ld32(tS + c * 32, chunk);
        }
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(&bar_s_free[slot]);
        ++cs;

        // Row max of the raw scores in 8 independent chains (three-input max:
        // two new scores per instruction); the causal mask only exists on the
        // diagonal tile (warp-uniform branch).
        const bool diag = (j == nkv - 1);
        if (diag) {
          const int lim = qrow - j * kBN;  // keys 0..lim of this tile are visible
#pragma unroll
          for (int c = 0; c < kBN; ++c)
            if (c > lim) sv[c] = __float_as_uint(-INFINITY);
        }
        float mx8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) mx8[i] = __uint_as_float(sv[i]);
#pragma unroll
        for (int c = 8; c < kBN; c += 16) {
#pragma unroll
          for (int i = 0; i < 8; ++i)
            mx8[i] = fmax3(mx8[i], __uint_as_float(sv[c + i]), __uint_as_float(sv[c + 8 + i]));
        }
        const float mx2 =
            fmax3(fmax3(mx8[0], mx8[1], mx8[2]), fmax3(mx8[3], mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])) *
            p.scale_log2;
        // Lazy rescaling: the running reference max m (log2 units) only moves
        // when the tile max exceeds it by more than 8, so P <= 2^8 and O is
        // rescaled only on those (rare after the first tiles) occasions.
        float alpha = 1.f;
        if (mx2 > m + 8.f) {
          alpha = (m == -INFINITY) ? 0.f : fast_exp2(m - mx2);
          m = mx2;
        }
        const float2 sc2 = make_float2(p.scale_log2, p.scale_log2);
        const float2 nm2 = make_float2(-m, -m);

        // P = exp2(s * scale_log2 - m) rounded to T and packed two per word, all
        // in registers: this does not touch the P tile, so it overlaps the P V
        // product of the previous tile.
        uint32_t pk[kBN / 2];
        float2 sum4[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) sum4[i] = make_float2(0.f, 0.f);
#pragma unroll
        for (int c = 0; c < kBN; c += 2) {
          const float2 x = fma2(make_float2(__uint_as_float(sv[c]), __uint_as_float(sv[c + 1])), sc2, nm2);
          const float2 e =
              ((c >> 1) & 7) < kPolyPairs ? exp2_poly2(x) : make_float2(fast_exp2(x.x), fast_exp2(x.y));
          sum4[(c >> 1) & 3] = add2(sum4[(c >> 1) & 3], e);
          pk[c >> 1] = pack2<T>(e.x, e.y);
        }
        const float2 s01 = add2(add2(sum4[0], sum4[1]), add2(sum4[2], sum4[3]));
        l = l * alpha + (s01.x + s01.y);

        if (j > 0) {
          // P V of the previous tile must be finished before the P tile is
          // overwritten and O is rescaled.  (Before an item's first tile the
          // previous item's epilogue has already waited for its last P V.)
          if (!__all_sync(0xffffffffu, wait_bounded(wc, &bar_o_done[slot], (cp - 1) & 1, 9))) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
#pragma unroll
        for (int ch = 0; ch < kBN / 32; ++ch)
          tmem_st16(tP + ch * 16, *reinterpret_cast<uint32_t(*)[16]>(&pk[ch * 16]));
        if (j > 0 && __any_sync(0xffffffffu, alpha < 1.f)) {
#pragma unroll
          for (int c = 0; c < D / 16; ++c) {
            uint32_t ov[16];
            tmem_ld16(tO + c * 16, ov);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
            tmem_st16(tO + c * 16, ov);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&bar_p_full[slot]);
        ++cp;
      }
      // epilogue: O / l -> global, logsumexp (natural log of scaled scores).
      // O is read completely before this slot's next P tile is announced, so
      // the next item's first P V (which overwrites O) cannot overtake it.
      if (!ok || !__all_sync(0xffffffffu, wait_bounded(wc, &bar_o_done[slot], (cp - 1) & 1, 10))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float inv_l = 1.f / l;
      T* orow = static_cast<T*>(p.o) + int64_t(w.b) * p.os[0] + int64_t(w.h) * p.os[1] + int64_t(qrow) * p.os[2];
#pragma unroll
      for (int c = 0; c < D / 16; ++c) {
        uint32_t ov[16];
        tmem_ld16(tO + c * 16, ov);
        tmem_ld_wait();
        if (qrow < p.T) {
          uint4 w0, w1;
          w0.x = pack2<T>(__uint_as_float(ov[0]) * inv_l, __uint_as_float(ov[1]) * inv_l);
          w0.y = pack2<T>(__uint_as_float(ov[2]) * inv_l, __uint_as_float(ov[3]) * inv_l);
          w0.z = pack2<T>(__uint_as_float(ov[4]) * inv_l, __uint_as_float(ov[5]) * inv_l);
          w0.w = pack2<T>(__uint_as_float(ov[6]) * inv_l, __uint_as_float(ov[7]) * inv_l);
          w1.x = pack2<T>(__uint_as_float(ov[8]) * inv_l, __uint_as_float(ov[9]) * inv_l);
          w1.y = pack2<T>(__uint_as_float(ov[10]) * inv_l, __uint_as_float(ov[11]) * inv_l);
          w1.z = pack2<T>(__uint_as_float(ov[12]) * inv_l, __uint_as_float(ov[13]) * inv_l);
          w1.w = pack2<T>(__uint_as_float(ov[14]) * inv_l, __uint_as_float(ov[15]) * inv_l);
          *reinterpret_cast<uint4*>(orow + c * 16) = w0;
          *reinterpret_cast<uint4*>(orow + c * 16 + 8) = w1;
        }
      }
      tc_fence_before();
      if (qrow < p.T)
        p.lse[(int64_t(w.b) * p.Hq + w.h) * p.T + qrow] = (m + __log2f(l)) * 0.69314718055994530942f;
    }
  }

  // teardown: every role reaches this point (bounded waits never hang)
  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

template <typename T, int D>
int launch_fwd(const FwdParams& prm, int B, int Hq, cudaStream_t stream) {
  using C = FwdCfg<D>;
  auto kern = attn_fwd_kernel<T, D>;
  int st = set_smem_limit((const void*)kern, C::SMEM);
  if (st != MT_OK) return st;
  cudaError_t err = cudaMemsetAsync(prm.sched, 0, sizeof(int), stream);  // work counter
  if (err != cudaSuccess) {
    set_last_error("cudaMemsetAsync", err);
    return MT_ERR_LAUNCH;
  }
  // persistent: one CTA per SM (the kernel's shared memory and TMEM allow one)
  const int blocks = prm.n_items < get_sm_count() ? prm.n_items : get_sm_count();
  record_timing_event(0, stream);
  kern<<<(unsigned)blocks, kThreads, C::SMEM, stream>>>(prm);
  record_timing_event(1, stream);
  return check_launch("attention_fwd");
}

}  // namespace

// Build a 4-D tensor map over a [B, H, T, D] tensor given element strides;
// the two middle dimensions are ordered by stride.  Returns MT status.
// swapped: -1 = choose from the strides (head stride below time stride, as in
// the model's [B, T, H, D] layout), else force the given order.
int make_bhtd_map(CUtensorMap* map, const void* base, int dtype, int64_t B, int64_t H, int64_t T, int64_t D,
                  const int64_t* s, int box_rows, int* swapped) {
  const int64_t es = 2;
  const bool sw = (*swapped >= 0) ? (*swapped != 0) : (s[1] < s[2]);
  uint64_t dims[4], strides[3];
  uint32_t box[4];
  dims[0] = D;
  box[0] = (uint32_t)D;
  if (sw) {
    dims[1] = H; dims[2] = T; strides[0] = s[1] * es; strides[1] = s[2] * es;
    box[1] = 1; box[2] = (uint32_t)box_rows;
  } else {
    dims[1] = T; dims[2] = H; strides[0] = s[2] * es; strides[1] = s[1] * es;
    box[1] = (uint32_t)box_rows; box[2] = 1;
  }
  dims[3] = B;
  strides[2] = s[0] * es;
  box[3] = 1;
  *swapped = sw ? 1 : 0;
  const CUtensorMapDataType dt = dtype == MT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const CUtensorMapSwizzle swz = D == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  return encode_tensor_map(map, dt, 4, const_cast<void*>(base), dims, strides, box, swz);
}

// Shared validation for the attention entry points.
int check_attn_layout(const void* ptr, const int64_t* s, bool need) {
  if (!need) return MT_OK;
  if (ptr == nullptr || s == nullptr) return MT_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(ptr) & 15u) != 0) return MT_ERR_UNSUPPORTED_LAYOUT;
  if (s[3] != 1) return MT_ERR_UNSUPPORTED_LAYOUT;
  for (int i = 0; i < 3; ++i)
    if (s[i] % 8 != 0 || s[i] <= 0) return MT_ERR_UNSUPPORTED_LAYOUT;
  return MT_OK;
}

}  // namespace mt

using namespace mt;

extern "C" int64_t mt_attention_fwd_workspace_bytes(int64_t B, int64_t Hq, int64_t T, int64_t D) {
  (void)B, (void)Hq, (void)T, (void)D;
  return 256;  // the persistent kernel's work counter
}

extern "C" int mt_attention_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int dtype,
                                int64_t B, int64_t Hq, int64_t Hkv, int64_t T, int64_t D, const int64_t* qs,
                                const int64_t* ks, const int64_t* vs, const int64_t* os, float scale,
                                void* workspace, int64_t workspace_bytes, uint32_t* status, void* stream) {
  if (dtype != MT_BF16 && dtype != MT_F16) return MT_ERR_UNSUPPORTED_DTYPE;
  if (B < 0 || Hq <= 0 || Hkv <= 0 || T < 0 || (Hq % Hkv) != 0) return MT_ERR_INVALID_ARGUMENT;
  if (D != 64 && D != 32) return MT_ERR_INVALID_ARGUMENT;
  if (B == 0 || T == 0) return MT_OK;
  if (lse == nullptr || status == nullptr) return MT_ERR_INVALID_ARGUMENT;
  if (B * Hq > 0x7fffffff || T > (int64_t(1) << 30)) return MT_ERR_INVALID_ARGUMENT;
  if (workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) & 15u) != 0 ||
      workspace_bytes < mt_attention_fwd_workspace_bytes(B, Hq, T, D))
    return MT_ERR_WORKSPACE;
  int st = MT_OK;
  if ((st = check_attn_layout(q, qs, true)) != MT_OK) return st;
  if ((st = check_attn_layout(k, ks, true)) != MT_OK) return st;
  if ((st = check_attn_layout(v, vs, true)) != MT_OK) return st;
  if ((st = check_attn_layout(o, os, true)) != MT_OK) return st;
  if ((st = bind_device_of(q)) != MT_OK) return st;
  if ((st = check_arch()) != MT_OK) return st;
  FwdParams prm;
  // One coordinate order per launch: chosen from q's strides, applied to k/v
  // (a size-1 head or time dimension makes either order valid).
  int swq = (Hq == 1 || T == 1) ? ((Hkv > 1 && T > 1) ? (ks[1] < ks[2] ? 1 : 0) : 0) : -1;
  if ((st = make_bhtd_map(&prm.tm_q, q, dtype, B, Hq, T, D, qs, kBM, &swq)) != MT_OK) return st;
  int swk = swq, swv = swq;
  if (Hkv > 1 && T > 1 && ((ks[1] < ks[2]) != (swq != 0) || (vs[1] < vs[2]) != (swq != 0)))
    return MT_ERR_UNSUPPORTED_LAYOUT;
  if ((st = make_bhtd_map(&prm.tm_k, k, dtype, B, Hkv, T, D, ks, kBN, &swk)) != MT_OK) return st;
  if ((st = make_bhtd_map(&prm.tm_v, v, dtype, B, Hkv, T, D, vs, kBN, &swv)) != MT_OK) return st;
  prm.ht_swapped = swq;
  prm.o = o;
  prm.lse = lse;
  for (int i = 0; i < 4; ++i) prm.os[i] = os[i];
  prm.T = (int)T;
  prm.Hq = (int)Hq;
  prm.Hkv = (int)Hkv;
  prm.repeats = (int)(Hq / Hkv);
  prm.n_qtiles = (int)((T + kBM - 1) / kBM);
  prm.n_pairs = (prm.n_qtiles + 1) / 2;
  if (B * Hq * prm.n_pairs > 0x7fffffff) return MT_ERR_INVALID_ARGUMENT;
  prm.n_items = (int)(B * Hq * prm.n_pairs);
  prm.scale_log2 = scale * 1.4426950408889634f;
  prm.status = status;
  prm.sched = static_cast<int*>(workspace);
  if (prm.n_qtiles > 65535) return MT_ERR_INVALID_ARGUMENT;
  auto s = static_cast<cudaStream_t>(stream);
  const bool bf = dtype == MT_BF16;
  if (D == 64) return bf ? launch_fwd<__nv_bfloat16, 64>(prm, (int)B, (int)Hq, s) : launch_fwd<__half, 64>(prm, (int)B, (int)Hq, s);
  return bf ? launch_fwd<__nv_bfloat16, 32>(prm, (int)B, (int)Hq, s) : launch_fwd<__half, 32>(prm, (int)B, (int)Hq, s);
}
