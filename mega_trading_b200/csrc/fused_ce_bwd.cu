// Fused linear + cross-entropy backward for sm_100a: dH = dZ W and
// dW = dZ^T H with the logit gradient dZ = (softmax(H W^T) - onehot) * g
// produced and consumed on chip, never written to global memory.
//
// Reference semantics (duoan/mega-trading): src/mega_trading/kernels/
// triton_ops.py:359-389 computes, per chunk of rows, grad_logits in place in
// the materialised logits chunk and then grad_hidden = dZ W and
// grad_weight += dZ^T H with two library GEMMs; g = grad_output / n_valid for
// rows whose label is not ignore_index, 0 otherwise (:330-357, :395-401).
//
// B200 design.  dH needs all vocab tiles of a row tile, dW all row tiles of a
// vocab tile, so the backward is two passes of one kernel template, each
// owning one output and recomputing the logit tiles it needs:
//   MODE 0 (dH): a cluster owns 128 rows and streams every 128-entry vocab
//                tile:   S = H_r W_j^T,  dZ,  dH_r += dZ W_j
//   MODE 1 (dW): a cluster owns 128 vocab entries and streams row tiles:
//                S^T = W_j H_r^T,  dZ^T,  dW_j += dZ^T H_r
// A 128 x 768 fp32 accumulator does not fit in one SM's TMEM next to the
// logit tile, so the output's hidden columns are split across the C CTAs of a
// thread-block cluster (C = ceil(H / 384), slices of <= 384 columns).  The C
// CTAs take turns computing the logit tile (each computes every C-th stream
// tile), round it to a 16-bit dZ tile in its own shared memory and push a copy
// into the others' shared memory with a DSMEM bulk copy
// (cp.async.bulk.shared::cluster.shared::cta, completing on the receiver's
// mbarrier); every CTA then multiplies every dZ tile by its slice of the
// stream operand.  So each logit is computed once per pass, and the logits
// cost 2 x 2NHV FLOP on top of the 2 x 2NHV of dH and dW.
//
// Per CTA: TMEM columns [0, 384) hold the output slice (fp32), [384, 512) the
// 128 x 128 logit tile.  Shared memory: C dZ slots of 32 KB (slot c is written
// by CTA c: a [128 x 128] 16-bit tile in the K-major 128B-swizzled layout the
// MMA's A operand reads) and a ring of 32 KB stages fed by TMA: for a logit
// tile, per 64-column K chunk, the fixed-side box and the stream-side box
// (K-major operands of S); for the output product, 128 output columns x the
// tile's 128 stream entities of a transposed copy of the stream operand (made
// by a transpose kernel in the workspace), so that both products read K-major
// operands (an MN-major B measured ~2x slower per instruction).  Warp roles (320 threads): warps 0-7 epilogue (thread =
// TMEM lane = fixed-side entity; warpgroup w takes logit columns [64w, 64w+64)
// and output panels p = w mod 2), warp 8 TMA producer + TMEM allocation,
// warp 9 MMA issuer.
//
// Issue order per CTA: S(own tile of round t+1), then the output products of
// round t's C tiles, so the epilogue of a logit tile overlaps the previous
// round's output products and the tensor pipe never waits for it.
// Synchronisation per dZ slot c: dz_full[c] (every CTA; the producer's
// epilogue arrives on its own copy, the bulk copy completes the bytes on the
// others' after their MMA thread armed the barrier), dz_free[c] (in CTA c; one
// tcgen05.commit arrival from each CTA's MMA thread, multicast to CTA c, when
// its products reading slot c are done).  Every wait is bounded.
#include <algorithm>
#include <type_traits>

#include "common.cuh"

namespace mt {
namespace {

constexpr int kT = 128;        // entities per tile
constexpr int kKC = 64;        // hidden columns per K chunk / output panel
constexpr int kBox = 16384;    // one [128 x 64] 16-bit box
constexpr int kStage = 32768;  // ring stage: two boxes
constexpr int kSlot = 32768;   // dZ tile [128 x 128] 16-bit
constexpr int kThreads = 320;
constexpr int kMaxSlice = 384;
constexpr int kMaxCluster = 3;
constexpr uint32_t kSCol = 384;  // TMEM column of the logit tile
constexpr uint32_t kKernelId = 4;

template <int C>
struct BwdCfg {
  static constexpr int NST = (224 * 1024 - C * kSlot) / kStage;  // C = 1, 2, 3: 6, 5, 4 stages
  static constexpr int OFF_SLOT = 0;
  static constexpr int OFF_STAGE = C * kSlot;
  static constexpr int OFF_BAR = OFF_STAGE + NST * kStage;
  static constexpr int OFF_RINFO = OFF_BAR + 512;  // MODE 1: per-column row inputs of the current tile
  static constexpr int SMEM = OFF_RINFO + kT * 16;
  static_assert(SMEM <= 227 * 1024, "shared memory");
};

struct BwdParams {
  CUtensorMap tm_f;  // fixed-side operand [f_count, K] (H for MODE 0, W for MODE 1), box 64 x 128
  CUtensorMap tm_x;  // stream-side operand [x_count, K], box 64 x 128
  CUtensorMap tm_xt; // its transpose [K, x_pad] (x_pad = x_count rounded to 8), box 64 x 128
  const float4* rinfo;  // per row: {-lse2, g, label bits, 0}; rows padded to a multiple of 128 with zeros
  int n_kc;             // 64-column chunks of K
  int f_count;          // entities of the fixed side
  int V;                // vocabulary size (entities beyond it are padding)
  int n_x_tiles;        // stream tiles in total
  int x_tiles_per_split;
  int slice_w;          // output columns per CTA (multiple of 64, <= 384)
  int stagger_mod, stagger_step;  // stream start of fixed tile y: (y % mod) * step tiles
  int hid0;             // first output column of this launch
  int hid_end;          // one past the last output column of this launch
  void* out;            // [f_count, out_ld] (+ split * split_stride): dH / dW or fp32 partials
  int out_dtype;
  int64_t out_ld;
  int64_t split_stride;
  uint32_t* status;
};

// DSMEM bulk copy of `bytes` from this CTA's shared memory to another CTA of
// the cluster; the bytes complete on the receiver's mbarrier.
__device__ __forceinline__ void bulk_copy_to_peer(uint32_t dst_cluster, const void* src, uint32_t bytes,
                                                  uint32_t bar_cluster) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   dst_cluster),
               "r"(smem_u32(src)), "r"(bytes), "r"(bar_cluster)
               : "memory");
}

// Arrive once on the mbarrier at this offset in every CTA of `cta_mask` when
// the MMAs issued so far by this thread have completed.
__device__ __forceinline__ void umma_commit_to(uint64_t* bar, uint16_t cta_mask) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
                   smem_u32(bar)),
               "h"(cta_mask)
               : "memory");
}

// 32 consecutive fp32 accumulator columns (raw TMEM words) -> dst[0, n_valid).
template <typename TO>
__device__ __forceinline__ void store_row32(TO* dst, const uint32_t (&v)[32], int n_valid) {
  if (n_valid >= 32 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
    constexpr int E = 16 / sizeof(TO);
#pragma unroll
    for (int i = 0; i < 32; i += E) {
      float q[E];
#pragma unroll
      for (int e = 0; e < E; ++e) q[e] = __uint_as_float(v[i + e]);
      store_vec<TO, E>(dst + i, q);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (i < n_valid) dst[i] = from_f32<TO>(__uint_as_float(v[i]));
  }
}

constexpr float kLog2e = 1.4426950408889634f;

// dZ of 32 logit columns of one row (MODE 0: thread = row, column = vocab
// entry x0 + i): (exp2(z log2e - lse2) - [x == label]) * g, 0 past the vocabulary.
template <typename T>
__device__ __forceinline__ void dz_cols_row(const uint32_t (&z)[32], int x0, int V, float nlse2, float g, int label,
                                            uint32_t (&pk)[16]) {
#pragma unroll
  for (int i = 0; i < 32; i += 2) {
    float d[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int x = x0 + i + e;
      const float pr = fast_exp2(fmaf(__uint_as_float(z[i + e]), kLog2e, nlse2));
      d[e] = x < V ? (pr - (x == label ? 1.f : 0.f)) * g : 0.f;
    }
    pk[i >> 1] = pack2<T>(d[0], d[1]);
  }
}

// dZ^T of 32 columns of one vocab entry v (MODE 1: thread = vocab entry,
// column i = row with inputs ri[i] = {-lse2, g, label} in shared memory).
template <typename T>
__device__ __forceinline__ void dz_cols_vocab(const uint32_t (&z)[32], const float4* ri, int v, bool v_ok,
                                              uint32_t (&pk)[16]) {
#pragma unroll
  for (int i = 0; i < 32; i += 2) {
    float d[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float4 q = ri[i + e];
      const float pr = fast_exp2(fmaf(__uint_as_float(z[i + e]), kLog2e, q.x));
      d[e] = v_ok ? (pr - (v == __float_as_int(q.z) ? 1.f : 0.f)) * q.y : 0.f;
    }
    pk[i >> 1] = pack2<T>(d[0], d[1]);
  }
}

template <typename T, int MODE, int C>
__global__ void __launch_bounds__(kThreads, 1) ce_bwd_kernel(const __grid_constant__ BwdParams p) {
  using Cfg = BwdCfg<C>;
  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = warp_id();
  const int lane = lane_id();
  if ((smem_u32(smem) & 1023u) != 0) {
    if (threadIdx.x == 0) atomicCAS(p.status, 0u, (kKernelId << 16) | 0xFFFFu);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::OFF_BAR);
  uint64_t* full = bars;                    // [NST]
  uint64_t* empty = bars + Cfg::NST;        // [NST]
  uint64_t* s_full = bars + 2 * Cfg::NST;   // logit tile computed
  uint64_t* s_free = s_full + 1;            // logit tile read out of TMEM
  uint64_t* acc_full = s_full + 2;          // every output product done
  uint64_t* fin = s_full + 3;               // MMA drain at exit
  uint64_t* dz_full = s_full + 4;           // [C]
  uint64_t* dz_free = dz_full + kMaxCluster;  // [C]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(dz_free + kMaxCluster);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);

  const int s = C > 1 ? (int)cluster_ctarank() : 0;
  const int f0 = blockIdx.y * kT;
  const int xs0 = blockIdx.z * p.x_tiles_per_split;
  const int xs1 = min(xs0 + p.x_tiles_per_split, p.n_x_tiles);
  const int n_x = max(xs1 - xs0, 0);
  const int n_rounds = (n_x + C - 1) / C;
  const int hid_base = p.hid0 + s * p.slice_w;
  const int n_panels = p.slice_w / kKC;
  const int n_ostages = (n_panels + 1) / 2;
  // clusters start their stream at staggered tiles (same order, rotated), so
  // the clusters resident at one time do not all read the same tile at once
  const int rot = n_x > 0 ? (int)(((int64_t)(blockIdx.y % p.stagger_mod) * p.stagger_step) % n_x) : 0;
  auto tile_of = [&](int t, int c) {
    int i = t * C + c + rot;
    if (i >= n_x) i -= n_x;
    return xs0 + i;
  };
  auto exists = [&](int t, int c) { return t < n_rounds && t * C + c < n_x; };

  if (threadIdx.x == 0) {
    for (int i = 0; i < Cfg::NST; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 256);
    mbar_init(acc_full, 1);
    mbar_init(fin, 1);
    for (int c = 0; c < C; ++c) {
      mbar_init(&dz_full[c], 1);
      mbar_init(&dz_free[c], C);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 8) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  if constexpr (C > 1)
    cluster_sync_all();  // every CTA's barriers exist before any copy or commit reaches them
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const WaitCtx wc{p.status, abort_flag, kKernelId};
  auto wait_x = [&](uint64_t* bar, uint32_t parity, uint32_t site) {
    if constexpr (C > 1)
      return wait_bounded_cluster(wc, bar, parity, site);
    else
      return wait_bounded(wc, bar, parity, site);
  };

  if (warp == 8) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&p.tm_f);
      tma_prefetch_desc(&p.tm_x);
      tma_prefetch_desc(&p.tm_xt);
      int it = 0;
      bool ok = true;
      auto next_stage = [&](uint32_t bytes) -> uint8_t* {
        const int st = it % Cfg::NST;
        if (it >= Cfg::NST && !wait_bounded(wc, &empty[st], ((it / Cfg::NST) & 1) ^ 1, 1)) {
          ok = false;
          return nullptr;
        }
        mbar_arrive_expect_tx(&full[st], bytes);
        return smem + Cfg::OFF_STAGE + st * kStage;
      };
      auto load_logits = [&](int xt) {
        for (int kc = 0; ok && kc < p.n_kc; ++kc) {
          uint8_t* sa = next_stage(kStage);
          if (!ok) break;
          tma_load_2d(sa, &p.tm_f, &full[it % Cfg::NST], kc * kKC, f0);
          tma_load_2d(sa + kBox, &p.tm_x, &full[it % Cfg::NST], kc * kKC, xt * kT);
          ++it;
        }
      };
      // the output product's B operand: 128 output columns x the tile's 128
      // stream entities, K-major from the transposed operand (two 64-entity atoms)
      auto load_panels = [&](int xt) {
        for (int q = 0; ok && q < n_ostages; ++q) {
          uint8_t* sa = next_stage(kStage);
          if (!ok) break;
          for (int e = 0; e < 2; ++e)
            tma_load_2d(sa + e * kBox, &p.tm_xt, &full[it % Cfg::NST], xt * kT + e * kKC, hid_base + q * 128);
          ++it;
        }
      };
      if (exists(0, s)) load_logits(tile_of(0, s));
      for (int t = 0; ok && t < n_rounds; ++t) {
        if (exists(t + 1, s)) load_logits(tile_of(t + 1, s));
        for (int c = 0; ok && c < C; ++c)
          if (exists(t, c)) load_panels(tile_of(t, c));
      }
      if (*abort_flag) {
        for (int j = (it > Cfg::NST ? it - Cfg::NST : 0); j < it; ++j)
          wait_drain(wc, &full[j % Cfg::NST], (j / Cfg::NST) & 1, 11);
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr int kBf16 = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
      constexpr uint32_t idesc_s = make_idesc(kT, kT, kBf16, 0, 0);
      const uint32_t slot_base = smem_u32(smem + Cfg::OFF_SLOT);
      const uint32_t stage_base = smem_u32(smem + Cfg::OFF_STAGE);
      int it = 0;
      int n_s = 0;  // logit tiles issued
      bool ok = true;
      bool first_out = true;
      int armed_round[kMaxCluster];  // last round whose peer dZ copy this CTA armed (-1: none)
      int done_round[kMaxCluster];   // last round whose dZ slot this CTA finished waiting for
      for (int c = 0; c < C; ++c) armed_round[c] = done_round[c] = -1;
      auto issue_logits = [&]() {
        if (n_s > 0 && !wait_bounded(wc, s_free, (n_s - 1) & 1, 2)) {
          ok = false;
          return;
        }
        tc_fence_after();
        for (int kc = 0; kc < p.n_kc; ++kc, ++it) {
          const int st = it % Cfg::NST;
          if (!wait_bounded(wc, &full[st], (it / Cfg::NST) & 1, 3)) {
            ok = false;
            return;
          }
          tc_fence_after();
          const uint32_t a = stage_base + st * kStage;
          // a K step of 16 elements advances the start address by 32 bytes (2 in the descriptor)
          const uint64_t da = make_sdesc(a, 16, 1024, kSwizzle128);
          const uint64_t db = make_sdesc(a + kBox, 16, 1024, kSwizzle128);
#pragma unroll
          for (int kk = 0; kk < kKC / 16; ++kk)
            umma_ss(tmem + kSCol, da + 2 * kk, db + 2 * kk, idesc_s, (kc > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&empty[st]);
        }
        umma_commit(s_full);
        ++n_s;
      };
      auto issue_out = [&](int t, int c) {
        if (c != s) {
          mbar_arrive_expect_tx(&dz_full[c], kSlot);  // the copy from CTA c completes these bytes
          armed_round[c] = t;
        }
        if (!wait_x(&dz_full[c], t & 1, 4)) {
          ok = false;
          return;
        }
        done_round[c] = t;
        tc_fence_after();
        const uint32_t a0 = slot_base + c * kSlot;
        for (int q = 0; q < n_ostages; ++q, ++it) {
          const int st = it % Cfg::NST;
          if (!wait_bounded(wc, &full[st], (it / Cfg::NST) & 1, 5)) {
            ok = false;
            return;
          }
          tc_fence_after();
          const int np = min(2, n_panels - 2 * q);
          const uint32_t idesc_o = make_idesc(kT, np * kKC, kBf16, 0, 0);
          const uint32_t b0 = stage_base + st * kStage;
          const uint64_t da[2] = {make_sdesc(a0, 16, 1024, kSwizzle128), make_sdesc(a0 + kBox, 16, 1024, kSwizzle128)};
          const uint64_t db[2] = {make_sdesc(b0, 16, 1024, kSwizzle128), make_sdesc(b0 + kBox, 16, 1024, kSwizzle128)};
#pragma unroll
          for (int kk = 0; kk < kT / 16; ++kk)
            umma_ss(tmem + q * 128, da[kk >> 2] + 2 * (kk & 3), db[kk >> 2] + 2 * (kk & 3), idesc_o,
                    (first_out && kk == 0) ? 0u : 1u);
          umma_commit(&empty[st]);
        }
        first_out = false;
        if constexpr (C > 1)
          umma_commit_to(&dz_free[c], (uint16_t)(1u << c));
        else
          umma_commit(&dz_free[c]);
      };
      if (exists(0, s)) issue_logits();
      for (int t = 0; ok && t < n_rounds; ++t) {
        if (exists(t + 1, s)) issue_logits();
        for (int c = 0; ok && c < C; ++c)
          if (exists(t, c)) issue_out(t, c);
      }
      if (ok) umma_commit(acc_full);
      if constexpr (C > 1) {
        if (!ok) {
          // a peer may still push the next dZ tile of each slot: let it land
          // before this CTA's shared memory goes away
          for (int c = 0; c < C; ++c) {
            if (c == s) continue;
            const int t = done_round[c] + 1;
            if (!exists(t, c)) continue;
            if (armed_round[c] < t) mbar_arrive_expect_tx(&dz_full[c], kSlot);
            wait_drain(wc, &dz_full[c], t & 1, 12);
          }
        }
      }
      umma_commit(fin);
      wait_drain(wc, fin, 0, 13);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int wg = warp >> 2;
    const int r = threadIdx.x & 127;  // TMEM lane = fixed-side entity of the tile
    const uint32_t lane_off = uint32_t((warp & 3) * 32) << 16;
    float4* ri_s = reinterpret_cast<float4*>(smem + Cfg::OFF_RINFO);
    // One thread polls a barrier while the other epilogue warps sleep in a
    // named barrier (polling warps would take issue slots from the MMA warp
    // on the same sub-partition); the poller's verdict reaches all 256.
    auto epi_wait = [&](auto&& wait_fn) -> bool {
      const bool v = threadIdx.x == 0 ? wait_fn() : true;
      return bar_all(v, 3, 256);
    };
    const int fe = f0 + r;  // this thread's fixed-side entity
    // MODE 0: the thread's row; MODE 1: the thread's vocab entry
    float nlse2 = 0.f, g = 0.f;
    int label = -1;
    if constexpr (MODE == 0) {
      if (fe < p.f_count) {
        const float4 ri = p.rinfo[fe];
        nlse2 = ri.x;
        g = ri.y;
        label = __float_as_int(ri.z);
      }
    }
    const bool fe_ok = MODE == 0 ? true : fe < p.V;
    uint8_t* my_slot = smem + Cfg::OFF_SLOT + s * kSlot;
    bool ok = true;
    int n_own = 0;
    for (int t = 0; t < n_rounds; ++t) {
      if (!exists(t, s)) break;
      const int xt = tile_of(t, s);
      if (!epi_wait([&] { return wait_bounded(wc, s_full, n_own & 1, 8); })) {
        ok = false;
        break;
      }
      tc_fence_after();
      if constexpr (MODE == 1) {
        // the tile's 128 rows: {-lse2, g, label} per column, read as broadcasts below
        if (threadIdx.x < kT) ri_s[threadIdx.x] = p.rinfo[xt * kT + threadIdx.x];
      }
      uint32_t z0[32], z1[32];
      tmem_ld32(tmem + lane_off + kSCol + wg * 64, z0);
      tmem_ld32(tmem + lane_off + kSCol + wg * 64 + 32, z1);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(s_free);
      if constexpr (MODE == 1) named_bar_sync(2, 256);
      const int x_base = xt * kT + wg * 64;  // stream-side entity of column 0 of this warpgroup
      uint32_t pk0[16], pk1[16];
      if constexpr (MODE == 0) {
        dz_cols_row<T>(z0, x_base, p.V, nlse2, g, label, pk0);
        dz_cols_row<T>(z1, x_base + 32, p.V, nlse2, g, label, pk1);
      } else {
        dz_cols_vocab<T>(z0, ri_s + wg * 64, fe, fe_ok, pk0);
        dz_cols_vocab<T>(z1, ri_s + wg * 64 + 32, fe, fe_ok, pk1);
      }
      // the slot's previous tile must be consumed by every CTA of the cluster
      if (n_own > 0 && !epi_wait([&] { return wait_x(&dz_free[s], (n_own - 1) & 1, 9); })) {
        ok = false;
        break;
      }
      // K-major 128B-swizzled: atom wg holds columns [64 wg, 64 wg + 64)
      uint8_t* row_base = my_slot + wg * kBox + r * 128;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        *reinterpret_cast<uint4*>(row_base + ((j ^ (r & 7)) << 4)) =
            make_uint4(pk0[4 * j], pk0[4 * j + 1], pk0[4 * j + 2], pk0[4 * j + 3]);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        *reinterpret_cast<uint4*>(row_base + (((j + 4) ^ (r & 7)) << 4)) =
            make_uint4(pk1[4 * j], pk1[4 * j + 1], pk1[4 * j + 2], pk1[4 * j + 3]);
      fence_proxy_async_smem();
      named_bar_sync(1, 256);
      if (threadIdx.x == 0) {
        mbar_arrive(&dz_full[s]);
        if constexpr (C > 1) {
          for (int c = 0; c < C; ++c)
            if (c != s)
              bulk_copy_to_peer(cluster_addr(my_slot, (uint32_t)c), my_slot, kSlot,
                                cluster_addr(&dz_full[s], (uint32_t)c));
        }
      }
      ++n_own;
    }
    // every CTA has finished with this CTA's last dZ tile: no copy or commit
    // addressed to this CTA is still in flight when it exits
    if (n_own > 0 && threadIdx.x == 0) wait_drain(wc, &dz_free[s], (n_own - 1) & 1, 10);
    if (ok && !*abort_flag && n_x > 0) {
      if (epi_wait([&] { return wait_bounded(wc, acc_full, 0, 6); })) {
        tc_fence_after();
        const bool store = fe < p.f_count && fe_ok;
        char* out_row = static_cast<char*>(p.out) +
                        ((int64_t)blockIdx.z * p.split_stride + (int64_t)(store ? fe : 0) * p.out_ld) *
                            (p.out_dtype == MT_F32 ? 4 : 2);
        for (int hc = wg; hc < 2 * n_panels; hc += 2) {
          // 32-column chunks; warp-collective TMEM loads: every lane takes part,
          // only rows that exist store
          uint32_t v[32];
          tmem_ld32(tmem + lane_off + hc * 32, v);
          tmem_ld_wait();
          const int h0 = hid_base + hc * 32;
          const int nv = p.hid_end - h0;
          if (!store || nv <= 0) continue;
          if (p.out_dtype == MT_F32)
            store_row32<float>(reinterpret_cast<float*>(out_row) + h0, v, nv);
          else if (p.out_dtype == MT_BF16)
            store_row32<__nv_bfloat16>(reinterpret_cast<__nv_bfloat16*>(out_row) + h0, v, nv);
          else
            store_row32<__half>(reinterpret_cast<__half*>(out_row) + h0, v, nv);
        }
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  if constexpr (C > 1)
    cluster_sync_all();  // no CTA leaves while another may still address its shared memory
  else
    __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Per-row inputs of both passes: {-lse2, g, label, 0} with g = grad_out / n_valid
// for rows with a valid label (0 otherwise); padded rows are all zero.
__global__ void ce_rowinfo_kernel(const void* __restrict__ labels, int labels_i64, int64_t ignore_index, int N,
                                  int Np, int V, const float* __restrict__ lse2, const float* __restrict__ scal,
                                  const float* __restrict__ grad_out, float4* __restrict__ rinfo) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= Np) return;
  float4 o = make_float4(0.f, 0.f, __int_as_float(-1), 0.f);
  if (row < N) {
    const int64_t label = labels_i64 ? static_cast<const int64_t*>(labels)[row]
                                     : (int64_t) static_cast<const int32_t*>(labels)[row];
    const bool valid = label != ignore_index && label >= 0 && label < V;
    o.x = -lse2[row];
    o.y = valid ? scal[2] * grad_out[0] : 0.f;
    o.z = __int_as_float(valid ? (int)label : -1);
  }
  rinfo[row] = o;
}

// out[f, h] = sum over splits of part[split, f, h] (fixed order), cast to out's dtype.
template <typename TO>
__global__ void ce_reduce_splits_kernel(const float* __restrict__ part, int splits, int64_t split_stride,
                                        int64_t rows, int K, TO* __restrict__ out) {
  const int64_t n4 = rows * K / 4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    float4 acc = reinterpret_cast<const float4*>(part)[i];
    for (int sp = 1; sp < splits; ++sp) {
      const float4 q = reinterpret_cast<const float4*>(part + sp * split_stride)[i];
      acc.x += q.x;
      acc.y += q.y;
      acc.z += q.z;
      acc.w += q.w;
    }
    const float v[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) out[4 * i + e] = from_f32<TO>(v[e]);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct SliceGroup {
  int hid0, hid_count, C, slice_w;
};

// Hidden columns are covered by groups of at most 3 x 384 columns; a group's
// columns are split into C slices of slice_w (a multiple of 64).
int slice_groups(int64_t K, SliceGroup* out, int max_groups) {
  int n = 0;
  for (int64_t h = 0; h < K; h += kMaxCluster * kMaxSlice) {
    if (n >= max_groups) return -1;
    const int hg = (int)std::min<int64_t>(K - h, kMaxCluster * kMaxSlice);
    const int C = (hg + kMaxSlice - 1) / kMaxSlice;
    const int per = (hg + C - 1) / C;
    out[n++] = SliceGroup{(int)h, hg, C, (per + kKC - 1) / kKC * kKC};
  }
  return n;
}

// Splits of the stream dimension: enough clusters to fill the GPU in whole
// waves, weighed against the fp32 partials each extra split writes and reads.
int choose_splits(int64_t fixed_tiles, int64_t stream_tiles, int C, double flops, double partial_bytes) {
  const int64_t resident = std::max<int64_t>(1, get_sm_count() / C);
  const double t_flops = flops / 1.1e15;
  int best = 1;
  double best_cost = 1e30;
  const int max_s = (int)std::max<int64_t>(1, std::min<int64_t>(16, stream_tiles / (2 * C)));
  for (int sp = 1; sp <= max_s; ++sp) {
    const int64_t clusters = fixed_tiles * sp;
    const int64_t waves = (clusters + resident - 1) / resident;
    const double eff = double(clusters) / double(waves * resident);
    const double cost = t_flops / eff + (sp > 1 ? double(sp) * partial_bytes * 2.0 / 6.0e12 : 0.0);
    if (cost < best_cost * 0.995) {
      best_cost = cost;
      best = sp;
    }
  }
  return best;
}

struct BwdPlan {
  int64_t Np;
  int splits[2];  // MODE 0 (dH), MODE 1 (dW)
  int64_t rinfo_bytes, part_bytes, xt_bytes, bytes;
};

BwdPlan plan_bwd(int64_t N, int64_t V, int64_t K) {
  BwdPlan pl;
  pl.Np = (N + kT - 1) / kT * kT;
  const int64_t row_tiles = pl.Np / kT;
  const int64_t voc_tiles = (V + kT - 1) / kT;
  const int C = (int)std::min<int64_t>(kMaxCluster, (K + kMaxSlice - 1) / kMaxSlice);
  const double flops = 4.0 * double(N) * double(V) * double(K);
  pl.splits[0] = choose_splits(row_tiles, voc_tiles, C, flops, double(pl.Np) * K * 4);
  pl.splits[1] = choose_splits(voc_tiles, row_tiles, C, flops, double(voc_tiles * kT) * K * 4);
  auto up = [](int64_t x) { return (x + 255) / 256 * 256; };
  pl.rinfo_bytes = up(pl.Np * 16);
  const int64_t p0 = pl.splits[0] > 1 ? int64_t(pl.splits[0]) * pl.Np * K * 4 : 0;
  const int64_t p1 = pl.splits[1] > 1 ? int64_t(pl.splits[1]) * voc_tiles * kT * K * 4 : 0;
  pl.part_bytes = up(std::max(p0, p1));
  // transposed stream operand of either pass (one at a time): [K, entities rounded to 128]
  pl.xt_bytes = up(K * std::max(pl.Np, voc_tiles * kT) * 2);
  pl.bytes = pl.rinfo_bytes + pl.part_bytes + pl.xt_bytes + 256;
  return pl;
}

// out[k, r] = in[r, k] for r < rows, 0 for rows <= r < ld_out (64 x 64 tiles through shared memory).
template <typename T>
__global__ void __launch_bounds__(256) transpose_kernel(const T* __restrict__ in, int64_t rows, int64_t K,
                                                        T* __restrict__ out, int64_t ld_out) {
  __shared__ T tile[64][66];
  const int64_t r0 = int64_t(blockIdx.x) * 64, k0 = int64_t(blockIdx.y) * 64;
  const int tx = threadIdx.x & 63, ty = threadIdx.x >> 6;  // 64 x 4 threads
  for (int i = ty; i < 64; i += 4) {
    const int64_t r = r0 + i, k = k0 + tx;
    tile[i][tx] = (r < rows && k < K) ? in[r * K + k] : from_f32<T>(0.f);
  }
  __syncthreads();
  for (int i = ty; i < 64; i += 4) {
    const int64_t k = k0 + i, r = r0 + tx;
    if (k < K && r < ld_out) out[k * ld_out + r] = tile[tx][i];
  }
}

int map_rows(CUtensorMap* m, int dtype, const void* base, int64_t rows, int64_t K) {
  const CUtensorMapDataType dt = dtype == MT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  uint64_t dims[2] = {(uint64_t)K, (uint64_t)rows};
  uint64_t str[1] = {(uint64_t)K * 2};
  uint32_t box[2] = {kKC, kT};
  return encode_tensor_map(m, dt, 2, const_cast<void*>(base), dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

template <typename T, int MODE, int C>
int launch_pass(BwdParams& prm, int64_t fixed_tiles, int splits, cudaStream_t stream) {
  using Cfg = BwdCfg<C>;
  auto kern = ce_bwd_kernel<T, MODE, C>;
  int st = set_smem_limit((const void*)kern, Cfg::SMEM);
  if (st != MT_OK) return st;
  if (fixed_tiles > 65535 || splits > 65535) return MT_ERR_INVALID_ARGUMENT;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)C, (unsigned)fixed_tiles, (unsigned)splits);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = Cfg::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t err = cudaLaunchKernelEx(&cfg, kern, prm);
  if (err != cudaSuccess) {
    set_last_error(MODE == 0 ? "fused_ce_bwd_dh" : "fused_ce_bwd_dw", err);
    return MT_ERR_LAUNCH;
  }
  return check_launch(MODE == 0 ? "fused_ce_bwd_dh" : "fused_ce_bwd_dw");
}

template <typename T, int MODE>
int launch_pass_c(BwdParams& prm, int C, int64_t fixed_tiles, int splits, cudaStream_t stream) {
  switch (C) {
    case 1: return launch_pass<T, MODE, 1>(prm, fixed_tiles, splits, stream);
    case 2: return launch_pass<T, MODE, 2>(prm, fixed_tiles, splits, stream);
    case 3: return launch_pass<T, MODE, 3>(prm, fixed_tiles, splits, stream);
    default: return MT_ERR_INVALID_ARGUMENT;
  }
}

int reduce_splits(const float* part, int splits, int64_t split_stride, int64_t rows, int64_t K, void* out,
                  int out_dtype, cudaStream_t s) {
  const int64_t n4 = rows * K / 4;
  const int blocks = (int)std::min<int64_t>((n4 + 255) / 256, int64_t(get_sm_count()) * 8);
  if (out_dtype == MT_F32)
    ce_reduce_splits_kernel<float><<<blocks, 256, 0, s>>>(part, splits, split_stride, rows, (int)K,
                                                           static_cast<float*>(out));
  else if (out_dtype == MT_BF16)
    ce_reduce_splits_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(part, splits, split_stride, rows, (int)K,
                                                                   static_cast<__nv_bfloat16*>(out));
  else
    ce_reduce_splits_kernel<__half><<<blocks, 256, 0, s>>>(part, splits, split_stride, rows, (int)K,
                                                            static_cast<__half*>(out));
  return check_launch("fused_ce_bwd_reduce");
}

// One pass (MODE 0: dH, MODE 1: dW) over every slice group of the hidden columns.
template <typename T, int MODE>
int run_pass(const BwdPlan& pl, const void* fixed, int64_t f_count, const void* stream_op, int64_t x_count, void* xt,
             int dtype, int64_t V, int64_t K, const float4* rinfo, float* part, void* out, int out_dtype,
             uint32_t* status, cudaStream_t s) {
  BwdParams prm;
  int st = map_rows(&prm.tm_f, dtype, fixed, f_count, K);
  if (st != MT_OK) return st;
  if ((st = map_rows(&prm.tm_x, dtype, stream_op, x_count, K)) != MT_OK) return st;
  // the output products read the stream operand K-major: a transposed copy
  const int64_t x_pad = (x_count + kT - 1) / kT * kT;
  {
    dim3 grid((unsigned)(x_pad / 64), (unsigned)((K + 63) / 64));
    transpose_kernel<T><<<grid, 256, 0, s>>>(static_cast<const T*>(stream_op), x_count, K, static_cast<T*>(xt),
                                              x_pad);
    if ((st = check_launch("fused_ce_bwd_transpose")) != MT_OK) return st;
    if ((st = map_rows(&prm.tm_xt, dtype, xt, K, x_pad)) != MT_OK) return st;
  }
  const int64_t fixed_tiles = (f_count + kT - 1) / kT;
  const int64_t x_tiles = (x_count + kT - 1) / kT;
  const int64_t per_split = (x_tiles + pl.splits[MODE] - 1) / pl.splits[MODE];
  // no split without stream tiles: every partial the reduction reads is written
  const int splits = (int)((x_tiles + per_split - 1) / per_split);
  prm.rinfo = rinfo;
  prm.n_kc = (int)((K + kKC - 1) / kKC);
  prm.f_count = (int)f_count;
  prm.V = (int)V;
  prm.n_x_tiles = (int)x_tiles;
  prm.x_tiles_per_split = (int)per_split;
  // All clusters stream in the same order (no stagger): measured at config 2,
  // spreading the starts over the weight (dH pass) or a 16-tile window of the
  // hidden states (dW pass) ran no faster and multiplied the DRAM reads
  // (0.16 -> 3.5 GB and 0.34 -> 0.71 GB per launch), the resident clusters no
  // longer sharing each tile in L2.
  prm.stagger_mod = 1;
  prm.stagger_step = 0;
  prm.status = status;
  const int64_t f_pad = fixed_tiles * kT;
  if (splits > 1) {
    prm.out = part;
    prm.out_dtype = MT_F32;
    prm.out_ld = K;
    prm.split_stride = f_pad * K;
  } else {
    prm.out = out;
    prm.out_dtype = out_dtype;
    prm.out_ld = K;
    prm.split_stride = 0;
  }
  SliceGroup groups[64];
  const int ng = slice_groups(K, groups, 64);
  if (ng < 0) return MT_ERR_UNSUPPORTED_LAYOUT;
  for (int gi = 0; gi < ng; ++gi) {
    prm.hid0 = groups[gi].hid0;
    prm.hid_end = groups[gi].hid0 + groups[gi].hid_count;
    prm.slice_w = groups[gi].slice_w;
    if ((st = launch_pass_c<T, MODE>(prm, groups[gi].C, fixed_tiles, splits, s)) != MT_OK) return st;
  }
  if (splits > 1) return reduce_splits(part, splits, f_pad * K, f_count, K, out, out_dtype, s);
  return MT_OK;
}

}  // namespace
}  // namespace mt

using namespace mt;

extern "C" int64_t mt_fused_ce_bwd_workspace_bytes(int64_t N, int64_t V, int64_t K) {
  if (N <= 0 || V <= 0 || K <= 0) return 256;
  return plan_bwd(N, V, K).bytes;
}

extern "C" int mt_fused_ce_bwd(const void* hidden, const void* weight, const void* labels, int labels_i64,
                               int64_t ignore_index, int dtype, int64_t N, int64_t V, int64_t K,
                               const float* lse2_scal, const float* grad_out, void* dhidden, int dh_dtype,
                               void* dweight, int dw_dtype, void* workspace, int64_t workspace_bytes,
                               uint32_t* status, void* stream) {
  if (dtype != MT_BF16 && dtype != MT_F16) return MT_ERR_UNSUPPORTED_DTYPE;
  if (N < 0 || V <= 0 || K <= 0) return MT_ERR_INVALID_ARGUMENT;
  if (N > 0x7fffffffLL - kT || V > 0x7fffffffLL - kT || K > 0x7fffffffLL / 4) return MT_ERR_INVALID_ARGUMENT;
  if (N > 0 && (hidden == nullptr || weight == nullptr || labels == nullptr)) return MT_ERR_INVALID_ARGUMENT;
  for (int od : {dh_dtype, dw_dtype})
    if (od != MT_F32 && od != MT_BF16 && od != MT_F16) return MT_ERR_UNSUPPORTED_DTYPE;
  if (K % 8 != 0) return MT_ERR_UNSUPPORTED_LAYOUT;
  if ((reinterpret_cast<uintptr_t>(hidden) & 15u) || (reinterpret_cast<uintptr_t>(weight) & 15u))
    return MT_ERR_UNSUPPORTED_LAYOUT;
  for (const void* o : {dhidden, dweight})
    if (o != nullptr && (reinterpret_cast<uintptr_t>(o) & 15u)) return MT_ERR_UNSUPPORTED_LAYOUT;
  auto s = static_cast<cudaStream_t>(stream);
  if (N == 0) {
    if (dweight != nullptr) {
      cudaError_t e = cudaMemsetAsync(dweight, 0, size_t(V) * K * (dw_dtype == MT_F32 ? 4 : 2), s);
      if (e != cudaSuccess) {
        set_last_error("cudaMemsetAsync(dweight)", e);
        return MT_ERR_LAUNCH;
      }
    }
    return MT_OK;
  }
  if (lse2_scal == nullptr || grad_out == nullptr || status == nullptr || workspace == nullptr)
    return MT_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return MT_ERR_WORKSPACE;
  int st = bind_device_of(hidden);
  if (st != MT_OK) return st;
  if ((st = check_arch()) != MT_OK) return st;
  const BwdPlan pl = plan_bwd(N, V, K);
  if (workspace_bytes < pl.bytes) return MT_ERR_WORKSPACE;
  char* ws = static_cast<char*>(workspace);
  float4* rinfo = reinterpret_cast<float4*>(ws);
  float* part = reinterpret_cast<float*>(ws + pl.rinfo_bytes);
  void* xt = ws + pl.rinfo_bytes + pl.part_bytes;
  ce_rowinfo_kernel<<<(unsigned)((pl.Np + 255) / 256), 256, 0, s>>>(labels, labels_i64, ignore_index, (int)N,
                                                                    (int)pl.Np, (int)V, lse2_scal, lse2_scal + N,
                                                                    grad_out, rinfo);
  if ((st = check_launch("fused_ce_bwd_rowinfo")) != MT_OK) return st;
  const bool bf = dtype == MT_BF16;
  if (dhidden != nullptr) {
    st = bf ? run_pass<__nv_bfloat16, 0>(pl, hidden, N, weight, V, xt, dtype, V, K, rinfo, part, dhidden, dh_dtype, status, s)
            : run_pass<__half, 0>(pl, hidden, N, weight, V, xt, dtype, V, K, rinfo, part, dhidden, dh_dtype, status, s);
    if (st != MT_OK) return st;
  }
  if (dweight != nullptr) {
    st = bf ? run_pass<__nv_bfloat16, 1>(pl, weight, V, hidden, N, xt, dtype, V, K, rinfo, part, dweight, dw_dtype, status, s)
            : run_pass<__half, 1>(pl, weight, V, hidden, N, xt, dtype, V, K, rinfo, part, dweight, dw_dtype, status, s);
    if (st != MT_OK) return st;
  }
  return MT_OK;
}
