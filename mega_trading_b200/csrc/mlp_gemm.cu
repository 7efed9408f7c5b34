// SwiGLU MLP projections as tcgen05 GEMMs with the gate fused into their
// epilogues, for sm_100a.
//
// Reference semantics (duoan/mega-trading): SwiGLU.forward
// src/mega_trading/model.py:249-256 -- w2(silu(w1(x)) * w3(x)) -- with the
// gate of kernels/triton_ops.py:57-61 (forward :774-782, backward :799-819):
// the projections are bf16 GEMMs (autocast) whose outputs are rounded to
// bf16, silu(gate) is rounded to the activation dtype before the product.
//
// B200 design
//   Both kernels are one persistent GEMM C[M, N] = A[M, K] B[N, K]^T (K-major
//   operands, 128B swizzle) over 128 x 256 tiles: a TMA producer warp streams
//   64-wide K chunks through an NST-stage ring, one thread issues
//   tcgen05.mma into one of two 256-column TMEM accumulators, and four
//   epilogue warps (thread = row = TMEM lane) drain the other accumulator in
//   32-column steps, so a tile's epilogue overlaps the next tile's MMAs.
//   Epilogue outputs leave through TMA stores of [128 x 32] 16-bit boxes.
//
//   MODE 0 (forward, W1||W3): B is the gate/up weight interleaved in blocks of
//     128 rows (w1[0:128], w3[0:128], w1[128:256], w3[128:256], ...), so each
//     256-column tile holds matching gate and up columns.  The epilogue writes
//     gate and up (rounded to bf16: the saved activation, in the same
//     interleaved layout) and y = round(round(silu(g)) * u), the W2 input.
//   MODE 1 (backward, W2 dgrad): A = dOut [M, H], B = W2^T [I, H]; the tile is
//     dY for 256 gate columns.  A loader warp prefetches the matching gate/up
//     boxes of the saved activation through a 3-slot ring; the epilogue rounds
//     dY to bf16 (the GEMM output dtype) and writes dgate / dup in the
//     interleaved layout: dg = dy u s (1 + g (1 - s)), du = dy round(g s).
//   MODE 2 (QKV projection + RoPE): B = [Wq; Wk; Wv]; the epilogue rounds the
//     projection to bf16 and rotates the q and k columns (the first rot_cols)
//     of the token at position t = row % T by the 16-bit RoPE tables
//     (interleaved pairs: (e c - o s, e s + o c), model.py:286-316), writing
//     the packed [q_rot | k_rot | v] rows attention reads in place.
// Warp roles (352 threads): warps 0-7 epilogue in two warpgroups taking
// alternate 32-column steps (each with its own staging boxes), 8 TMA producer
// (+ TMEM allocation), 9 MMA issuer, 10 epilogue-input loader (MODE 1).
//
// CTA pairs (PAIR: MODE 0 with M > 128): a cluster of two CTAs computes a
// 256 x 256 tile with tcgen05 cta_group::2 MMAs (M = 256).  Each CTA stages
// its own 128 A rows and one 128-row half of B (32 KB per stage instead of
// 48 KB: a single CTA streaming a whole 128 x 256 tile needs ~1.5x the
// shared-memory bandwidth the tensor core leaves for it), and holds its 128
// accumulator rows in its own TMEM.  Both CTAs' stage loads (cta_group::2
// TMA, each into its own CTA's memory) complete on the even CTA's full barrier, which expects
// both CTAs' bytes; the even CTA issues the MMAs and commits to both CTAs'
// empty / accumulator barriers (one commit with a two-CTA mask); both epilogues release the
// accumulator to the even CTA.  Before teardown the odd CTA waits (bounded)
// for the release of every stage it loaded, which the even CTA's MMAs can
// only signal after those bytes landed.  (MODE 1 is bound by its gate/up HBM
// traffic and MODE 2 measured faster unpaired, so they stay single-CTA.)
#include <algorithm>
#include <cmath>
#include <initializer_list>
#include <type_traits>

#include "common.cuh"

namespace mt {
namespace {

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 64;
constexpr int kEC = 32;    // epilogue columns per step
constexpr int kGB = 128;   // gate / up interleave block
constexpr int kThreads = 352;
constexpr uint32_t kKernelId = 6;

template <int MODE, bool PAIR>
struct GCfg {
  static constexpr int NST = PAIR ? (MODE == 0 ? 5 : (MODE == 1 ? 4 : 6)) : (MODE == 2 ? 4 : 3);
  static constexpr int TM = PAIR ? 2 * kBM : kBM;      // tile rows (the pair's M)
  static constexpr int B_ROWS = PAIR ? kBN / 2 : kBN;  // rows of B this CTA stages
  static constexpr int A_BYTES = kBM * kBK * 2;        // 16 KB
  static constexpr int B_BYTES = B_ROWS * kBK * 2;     // 16 KB (pair) or 32 KB
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int BOX = kBM * kEC * 2;      // [128 rows][32 cols] 16-bit = 8 KB, 64 B rows
  static constexpr int N_OUT = MODE == 0 ? 3 : (MODE == 1 ? 2 : 1);
  static constexpr int E = MODE == 1 ? 3 : 0;    // epilogue-input ring slots (gate + up box each)
  static constexpr int OFF_OUT = NST * STAGE;    // [2 warpgroups][N_OUT boxes]
  static constexpr int OFF_IN = OFF_OUT + 2 * N_OUT * BOX;
  static constexpr int OFF_BAR = OFF_IN + E * 2 * BOX;
  static constexpr int SMEM = OFF_BAR + 256;
  static_assert(E <= 8 && 2 * NST + 5 + 8 + E <= 28, "mbarriers overlap the TMEM slot");
  static_assert(SMEM <= 227 * 1024, "more shared memory than one sm_100 CTA may use");
};

struct GemmParams {
  CUtensorMap tm_a, tm_b;  // A [M, K], B [N, K]
  CUtensorMap tm_gu;       // saved gate/up [M, 2I] (MODE 0: stored, MODE 1: loaded), 32-column boxes
  CUtensorMap tm_out;      // MODE 0: y [M, I]; MODE 1: dgate/dup [M, 2I]; 32-column boxes
  int M, n_nt, n_tiles, n_k;
  // MODE 2: RoPE tables [T, head_dim / 2] (row stride rope_ld) and geometry
  const void* rope_cos;
  const void* rope_sin;
  int64_t rope_ld;
  int seq, head_dim, rot_cols;
  uint32_t* status;
};

// 64B-swizzled [rows][32] 16-bit box: byte offset of 16-byte chunk j of row r.
__device__ __forceinline__ int box_off(int r, int j) { return r * 64 + ((j ^ ((r >> 1) & 3)) << 4); }

template <typename T, int MODE, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1) mlp_gemm_kernel(const __grid_constant__ GemmParams p) {
  using C = GCfg<MODE, PAIR>;
  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = warp_id();
  const int lane = lane_id();
  if ((smem_u32(smem) & 1023u) != 0) {
    if (threadIdx.x == 0) atomicCAS(p.status, 0u, (kKernelId << 16) | 0xFFFFu);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* full = bars;                     // [NST]
  uint64_t* empty = bars + C::NST;           // [NST]
  uint64_t* acc_full = bars + 2 * C::NST;    // [2]
  uint64_t* acc_empty = acc_full + 2;        // [2]
  uint64_t* fin = acc_full + 4;
  uint64_t* in_full = fin + 1;               // [E]
  uint64_t* in_empty = in_full + 8;          // [E], E <= 8
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 28);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 29);

  // pair geometry: the even CTA (rank 0) leads; a "unit" is a pair or a lone CTA
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  const int unit = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int n_units = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  const int row_off = (int)rank * kBM;  // this CTA's first row inside a tile

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::NST; ++s) {
      // a pair's stage is full once the leader armed it and both CTAs' bytes landed
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&acc_full[s], 1);
      mbar_init(&acc_empty[s], PAIR ? 16 : 8);  // one arrival per epilogue warp (of both CTAs)
    }
    mbar_init(fin, 1);
    for (int s = 0; s < C::E; ++s) {
      mbar_init(&in_full[s], 1);
      mbar_init(&in_empty[s], 128);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 8) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, 512);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, 512);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (PAIR)
    cluster_sync_all();  // both CTAs' barriers exist before either signals the other
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const WaitCtx wc{p.status, abort_flag, kKernelId};
  // waits on barriers the partner CTA (or its tensor core) signals
  auto wait_x = [&](uint64_t* bar, uint32_t parity, uint32_t site) {
    if constexpr (PAIR)
      return wait_bounded_cluster(wc, bar, parity, site);
    else
      return wait_bounded(wc, bar, parity, site);
  };

  if (warp == 8) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&p.tm_a);
      tma_prefetch_desc(&p.tm_b);
      int it = 0;
      bool ok = true;
      for (int t = unit; ok && t < p.n_tiles; t += n_units) {
        const int mt = t / p.n_nt, nt = t - mt * p.n_nt;
        for (int kc = 0; kc < p.n_k; ++kc, ++it) {
          const int st = it % C::NST;
          if (it >= C::NST && !wait_x(&empty[st], ((it / C::NST) & 1) ^ 1, 1)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + st * C::STAGE;
          if constexpr (PAIR) {
            if (leader) mbar_arrive_expect_tx(&full[st], 2 * C::STAGE);
            const uint32_t bar = leader_addr(&full[st]);
            tma_load_2d_pair(sa, &p.tm_a, bar, kc * kBK, mt * C::TM + row_off);
            tma_load_2d_pair(sa + C::A_BYTES, &p.tm_b, bar, kc * kBK, nt * kBN + (int)rank * C::B_ROWS);
          } else {
            mbar_arrive_expect_tx(&full[st], C::STAGE);
            tma_load_2d(sa, &p.tm_a, &full[st], kc * kBK, mt * C::TM + row_off);
            tma_load_2d(sa + C::A_BYTES, &p.tm_b, &full[st], kc * kBK, nt * kBN + (int)rank * C::B_ROWS);
          }
        }
      }
      if (PAIR && !leader) {
        // the odd CTA's loads complete on the leader's barrier: wait until the
        // leader's MMAs released every stage loaded here (bounded)
        for (int j = (it > C::NST ? it - C::NST : 0); j < it; ++j)
          wait_drain(wc, &empty[j % C::NST], (j / C::NST) & 1, 15);
      }
      if (*abort_flag) {
        for (int j = (it > C::NST ? it - C::NST : 0); j < it; ++j) wait_drain(wc, &full[j % C::NST], (j / C::NST) & 1, 11);
      }
    }
  } else if (warp == 9 && PAIR && !leader) {
    // the odd CTA issues no MMAs
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr int kBf16 = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
      constexpr uint32_t idesc = make_idesc(C::TM, kBN, kBf16, 0, 0);
      const uint32_t base = smem_u32(smem);
      int it = 0, lt = 0;
      bool ok = true;
      for (int t = unit; ok && t < p.n_tiles; t += n_units, ++lt) {
        const int buf = lt & 1;
        if (lt >= 2 && !wait_x(&acc_empty[buf], ((lt >> 1) & 1) ^ 1, 2)) break;
        tc_fence_after();
        const uint32_t d = tmem + buf * kBN;
        for (int kc = 0; kc < p.n_k; ++kc, ++it) {
          const int st = it % C::NST;
          if (!wait_x(&full[st], (it / C::NST) & 1, 3)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = base + st * C::STAGE;
          const uint32_t b = a + C::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t ad = make_sdesc(a + kk * 32, 16, 1024, kSwizzle128);
            const uint64_t bd = make_sdesc(b + kk * 32, 16, 1024, kSwizzle128);
            if constexpr (PAIR)
              umma_ss_pair(d, ad, bd, idesc, (kc > 0 || kk > 0) ? 1u : 0u);
            else
              umma_ss(d, ad, bd, idesc, (kc > 0 || kk > 0) ? 1u : 0u);
          }
          if constexpr (PAIR)
            umma_commit_pair_mc(&empty[st], 3);
          else
            umma_commit(&empty[st]);
        }
        if (ok) {
          if constexpr (PAIR)
            umma_commit_pair_mc(&acc_full[buf], 3);
          else
            umma_commit(&acc_full[buf]);
        }
      }
      if constexpr (PAIR)
        umma_commit_pair(fin);
      else
        umma_commit(fin);
      wait_drain(wc, fin, 0, 13);
    }
  } else if (warp == 10) {
    // ------------------------------------------------------------ epilogue-input loader
    if constexpr (MODE == 1) {
      if (lane == 0) {
        tma_prefetch_desc(&p.tm_gu);
        int q = 0;
        bool ok = true;
        for (int t = unit; ok && t < p.n_tiles; t += n_units) {
          const int mt = t / p.n_nt, nt = t - mt * p.n_nt;
          for (int c = 0; c < kBN / kEC; ++c, ++q) {
            const int slot = q % C::E;
            if (q >= C::E && !wait_bounded(wc, &in_empty[slot], ((q / C::E) & 1) ^ 1, 4)) {
              ok = false;
              break;
            }
            const int col = nt * kBN + c * kEC;            // gate column index in [0, I)
            const int gcol = (col / kGB) * (2 * kGB) + (col % kGB);
            uint8_t* dst = smem + C::OFF_IN + slot * 2 * C::BOX;
            mbar_arrive_expect_tx(&in_full[slot], 2 * C::BOX);
            tma_load_2d(dst, &p.tm_gu, &in_full[slot], gcol, mt * C::TM + row_off);
            tma_load_2d(dst + C::BOX, &p.tm_gu, &in_full[slot], gcol + kGB, mt * C::TM + row_off);
          }
        }
        if (*abort_flag) {
          for (int j = (q > C::E ? q - C::E : 0); j < q; ++j) wait_drain(wc, &in_full[j % C::E], (j / C::E) & 1, 12);
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int wg = warp >> 2;            // takes the 32-column steps c with c % 2 == wg
    const int r = threadIdx.x & 127;     // row within the tile = TMEM lane
    const uint32_t lane_off = uint32_t((warp & 3) * 32) << 16;
    uint8_t* out = smem + C::OFF_OUT + wg * C::N_OUT * C::BOX;
    bool ok = true;
    int lt = 0;
    // the accumulator buffer is released by one arrival per warp (at the
    // leader's barrier for a pair)
    const uint32_t acc_empty_x[2] = {PAIR ? cluster_addr(&acc_empty[0], 0) : 0u,
                                     PAIR ? cluster_addr(&acc_empty[1], 0) : 0u};
    auto release_acc = [&](int b) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (PAIR)
          mbar_arrive_remote(acc_empty_x[b]);
        else
          mbar_arrive(&acc_empty[b]);
      }
    };
    for (int t = unit; ok && t < p.n_tiles; t += n_units, ++lt) {
      const int qt = lt * (kBN / kEC);  // MODE 1: first input-ring step of this tile
      const int mt = t / p.n_nt, nt = t - mt * p.n_nt;
      const int row0 = mt * C::TM + row_off;  // first row of this CTA's part of the tile
      const int buf = lt & 1;
      if (!__all_sync(0xffffffffu, wait_x(&acc_full[buf], (lt >> 1) & 1, 8))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t acc = tmem + lane_off + buf * kBN;
      if constexpr (MODE == 0) {
#pragma unroll 1
        for (int c = wg; c < kGB / kEC; c += 2) {
          uint32_t zg[32], zu[32];
          tmem_ld32(acc + c * kEC, zg);
          tmem_ld32(acc + kGB + c * kEC, zu);
          tmem_ld_wait();
          if (c + 2 >= kGB / kEC) release_acc(buf);
          uint32_t pg[16], pu[16], py[16];
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            // projections rounded to the activation dtype, as the GEMM output is
            const float g0 = round_epi<T>(__uint_as_float(zg[i])), g1 = round_epi<T>(__uint_as_float(zg[i + 1]));
            const float u0 = round_epi<T>(__uint_as_float(zu[i])), u1 = round_epi<T>(__uint_as_float(zu[i + 1]));
            pg[i >> 1] = pack_exact2<T>(g0, g1);
            pu[i >> 1] = pack_exact2<T>(u0, u1);
            py[i >> 1] = pack2<T>(round_epi<T>(g0 * sigmoid_f32(g0)) * u0, round_epi<T>(g1 * sigmoid_f32(g1)) * u1);
          }
          // this warpgroup's previous stores must have finished reading its staging boxes
          if (r == 0) bulk_wait_group_read0();
          named_bar_sync(1 + wg, 128);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            *reinterpret_cast<uint4*>(out + box_off(r, j)) = make_uint4(pg[j * 4], pg[j * 4 + 1], pg[j * 4 + 2], pg[j * 4 + 3]);
            *reinterpret_cast<uint4*>(out + C::BOX + box_off(r, j)) =
                make_uint4(pu[j * 4], pu[j * 4 + 1], pu[j * 4 + 2], pu[j * 4 + 3]);
            *reinterpret_cast<uint4*>(out + 2 * C::BOX + box_off(r, j)) =
                make_uint4(py[j * 4], py[j * 4 + 1], py[j * 4 + 2], py[j * 4 + 3]);
          }
          fence_proxy_async_smem();
          named_bar_sync(1 + wg, 128);
          if (r == 0) {
            const int gcol = nt * kBN + c * kEC;  // interleaved gate/up columns of this tile
            tma_store_2d(&p.tm_gu, out, gcol, row0);
            tma_store_2d(&p.tm_gu, out + C::BOX, gcol + kGB, row0);
            tma_store_2d(&p.tm_out, out + 2 * C::BOX, nt * kGB + c * kEC, row0);
            bulk_commit_group();
          }
        }
      } else if constexpr (MODE == 2) {
        const int row = row0 + r;
        const int t_pos = row % p.seq;
#pragma unroll 1
        for (int c = wg; c < kBN / kEC; c += 2) {
          uint32_t z[32];
          tmem_ld32(acc + c * kEC, z);
          tmem_ld_wait();
          if (c + 2 >= kBN / kEC) release_acc(buf);
          const int col0 = nt * kBN + c * kEC;
          uint32_t pk[16];
          if (col0 < p.rot_cols) {
            // pairs (2i, 2i+1) of this head: table entries i0 .. i0 + 15
            const int i0 = (col0 % p.head_dim) >> 1;
            const T* cp = static_cast<const T*>(p.rope_cos) + int64_t(t_pos) * p.rope_ld + i0;
            const T* sp = static_cast<const T*>(p.rope_sin) + int64_t(t_pos) * p.rope_ld + i0;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const uint4 cr = *reinterpret_cast<const uint4*>(cp + h * 8);
              const uint4 sr = *reinterpret_cast<const uint4*>(sp + h * 8);
              const uint32_t cw[4] = {cr.x, cr.y, cr.z, cr.w}, sw[4] = {sr.x, sr.y, sr.z, sr.w};
#pragma unroll
              for (int w = 0; w < 4; ++w) {
                float cs[2], sn[2];
                unpack2<T>(cw[w], cs[0], cs[1]);
                unpack2<T>(sw[w], sn[0], sn[1]);
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                  const int i = h * 8 + w * 2 + e;  // pair index within the chunk
                  const float ev = round_epi<T>(__uint_as_float(z[2 * i]));
                  const float od = round_epi<T>(__uint_as_float(z[2 * i + 1]));
                  pk[i] = pack2<T>(ev * cs[e] - od * sn[e], ev * sn[e] + od * cs[e]);
                }
              }
            }
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) pk[i] = pack2<T>(__uint_as_float(z[2 * i]), __uint_as_float(z[2 * i + 1]));
          }
          if (r == 0) bulk_wait_group_read0();
          named_bar_sync(1 + wg, 128);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            *reinterpret_cast<uint4*>(out + box_off(r, j)) = make_uint4(pk[j * 4], pk[j * 4 + 1], pk[j * 4 + 2], pk[j * 4 + 3]);
          fence_proxy_async_smem();
          named_bar_sync(1 + wg, 128);
          if (r == 0) {
            tma_store_2d(&p.tm_out, out, col0, row0);
            bulk_commit_group();
          }
        }
      } else {
#pragma unroll 1
        for (int c = wg; c < kBN / kEC; c += 2) {
          const int q = qt + c;  // step index across tiles, in the loader's order
          uint32_t zd[32];
          tmem_ld32(acc + c * kEC, zd);
          tmem_ld_wait();
          if (c + 2 >= kBN / kEC) release_acc(buf);
          const int slot = q % C::E;
          if (!__all_sync(0xffffffffu, wait_bounded(wc, &in_full[slot], (q / C::E) & 1, 9))) {
            ok = false;
            break;
          }
          const uint8_t* src = smem + C::OFF_IN + slot * 2 * C::BOX;
          uint32_t gw[16], uw[16];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint4 a = *reinterpret_cast<const uint4*>(src + box_off(r, j));
            const uint4 b = *reinterpret_cast<const uint4*>(src + C::BOX + box_off(r, j));
            gw[j * 4] = a.x; gw[j * 4 + 1] = a.y; gw[j * 4 + 2] = a.z; gw[j * 4 + 3] = a.w;
            uw[j * 4] = b.x; uw[j * 4 + 1] = b.y; uw[j * 4 + 2] = b.z; uw[j * 4 + 3] = b.w;
          }
          mbar_arrive(&in_empty[slot]);
          uint32_t pg[16], pu[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float g[2], u[2], o_g[2], o_u[2];
            unpack2<T>(gw[i], g[0], g[1]);
            unpack2<T>(uw[i], u[0], u[1]);
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const float dy = round_epi<T>(__uint_as_float(zd[2 * i + e]));  // dY is a bf16 GEMM output
              const float s = sigmoid_f32(g[e]);
              o_g[e] = dy * u[e] * s * (1.f + g[e] * (1.f - s));
              o_u[e] = dy * round_epi<T>(g[e] * s);
            }
            pg[i] = pack2<T>(o_g[0], o_g[1]);
            pu[i] = pack2<T>(o_u[0], o_u[1]);
          }
          if (r == 0) bulk_wait_group_read0();
          named_bar_sync(1 + wg, 128);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            *reinterpret_cast<uint4*>(out + box_off(r, j)) = make_uint4(pg[j * 4], pg[j * 4 + 1], pg[j * 4 + 2], pg[j * 4 + 3]);
            *reinterpret_cast<uint4*>(out + C::BOX + box_off(r, j)) =
                make_uint4(pu[j * 4], pu[j * 4 + 1], pu[j * 4 + 2], pu[j * 4 + 3]);
          }
          fence_proxy_async_smem();
          named_bar_sync(1 + wg, 128);
          if (r == 0) {
            const int col = nt * kBN + c * kEC;
            const int gcol = (col / kGB) * (2 * kGB) + (col % kGB);
            tma_store_2d(&p.tm_out, out, gcol, row0);
            tma_store_2d(&p.tm_out, out + C::BOX, gcol + kGB, row0);
            bulk_commit_group();
          }
        }
      }
    }
    // stores must finish reading shared memory before the CTA exits
    if (r == 0) bulk_wait_group0();
  }

  tc_fence_before();
  if constexpr (PAIR)
    cluster_sync_all();  // the leader's MMAs into this CTA are done; no arrival is still in flight
  else
    __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem, 512);
    else
      tmem_dealloc(tmem, 512);
  }
}

int map_2d(CUtensorMap* map, int dtype, const void* base, int64_t inner, int64_t outer, int64_t ld, uint32_t box_in,
           uint32_t box_out, CUtensorMapSwizzle swz) {
  const CUtensorMapDataType dt = dtype == MT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  uint64_t dims[2] = {(uint64_t)inner, (uint64_t)outer};
  uint64_t strides[1] = {(uint64_t)ld * 2};
  uint32_t box[2] = {box_in, box_out};
  return encode_tensor_map(map, dt, 2, const_cast<void*>(base), dims, strides, box, swz);
}

int validate(int dtype, int64_t M, int64_t K, int64_t I, std::initializer_list<const void*> ptrs) {
  if (dtype != MT_BF16 && dtype != MT_F16) return MT_ERR_UNSUPPORTED_DTYPE;
  if (M < 0 || K <= 0 || I <= 0) return MT_ERR_INVALID_ARGUMENT;
  if (I % kBN != 0 || K % 8 != 0) return MT_ERR_UNSUPPORTED_LAYOUT;  // whole 256-column tiles of gate columns
  if (M > 0x7fffffffLL - kBM || 2 * I > 0x7fffffffLL) return MT_ERR_INVALID_ARGUMENT;
  for (const void* q : ptrs)
    if (M > 0 && (q == nullptr || (reinterpret_cast<uintptr_t>(q) & 15u) != 0)) return MT_ERR_UNSUPPORTED_LAYOUT;
  return MT_OK;
}

// CTA pairs for the gate/up projection whenever the rows fill more than one
// 128-row tile.
bool use_pair(int MODE, int64_t M) { return MODE == 0 && M > kBM; }

template <int MODE, bool PAIR>
int launch_impl(GemmParams& prm, int dtype, int64_t M, int64_t K, int64_t N, cudaStream_t stream) {
  using C = GCfg<MODE, PAIR>;
  const int64_t n_mt = (M + C::TM - 1) / C::TM;
  prm.M = (int)M;
  prm.n_nt = (int)(N / kBN);
  prm.n_tiles = (int)(n_mt * prm.n_nt);
  prm.n_k = (int)((K + kBK - 1) / kBK);
  if (n_mt * prm.n_nt > 0x7fffffffLL) return MT_ERR_INVALID_ARGUMENT;
  const int per_unit = PAIR ? 2 : 1;
  const int units = (int)std::min<int64_t>(prm.n_tiles, get_sm_count() / per_unit);
  const bool bf = dtype == MT_BF16;
  auto kern = bf ? mlp_gemm_kernel<__nv_bfloat16, MODE, PAIR> : mlp_gemm_kernel<__half, MODE, PAIR>;
  int st = set_smem_limit((const void*)kern, C::SMEM);
  if (st != MT_OK) return st;
  const char* name = MODE == 0 ? "mlp_gemm_swiglu_fwd" : (MODE == 1 ? "mlp_gemm_swiglu_bwd" : "qkv_gemm_rope");
  if constexpr (PAIR) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(units * 2));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    // persistent: no more pairs than can be resident at once
    int resident = 0;
    if (cudaOccupancyMaxActiveClusters(&resident, kern, &cfg) == cudaSuccess && resident > 0 && resident < units)
      cfg.gridDim = dim3((unsigned)(resident * 2));
    cudaError_t err = cudaLaunchKernelEx(&cfg, kern, prm);
    if (err != cudaSuccess) {
      set_last_error(name, err);
      return MT_ERR_LAUNCH;
    }
  } else {
    kern<<<units, kThreads, C::SMEM, stream>>>(prm);
  }
  return check_launch(name);
}

template <int MODE>
int launch(GemmParams& prm, int dtype, int64_t M, int64_t K, int64_t N, cudaStream_t stream) {
  if constexpr (MODE == 0)
    if (use_pair(MODE, M)) return launch_impl<MODE, true>(prm, dtype, M, K, N, stream);
  return launch_impl<MODE, false>(prm, dtype, M, K, N, stream);
}
// B's tensor map box holds the rows one CTA stages: 256, or 128 for a pair.
uint32_t b_box_rows(int MODE, int64_t M) { return use_pair(MODE, M) ? kBN / 2 : kBN; }

}  // namespace
}  // namespace mt

using namespace mt;

extern "C" int mt_swiglu_gemm_fwd(const void* x, const void* w13, void* gu, void* y, int dtype, int64_t M, int64_t K,
                                  int64_t I, uint32_t* status, void* stream) {
  int st = validate(dtype, M, K, I, {x, w13, gu, y});
  if (st != MT_OK) return st;
  if (M == 0) return MT_OK;
  if (status == nullptr) return MT_ERR_INVALID_ARGUMENT;
  if ((st = bind_device_of(x)) != MT_OK) return st;
  if ((st = check_arch()) != MT_OK) return st;
  GemmParams prm;
  prm.status = status;
  if ((st = map_2d(&prm.tm_a, dtype, x, K, M, K, kBK, kBM, CU_TENSOR_MAP_SWIZZLE_128B)) != MT_OK) return st;
  if ((st = map_2d(&prm.tm_b, dtype, w13, K, 2 * I, K, kBK, b_box_rows(0, M), CU_TENSOR_MAP_SWIZZLE_128B)) != MT_OK)
    return st;
  if ((st = map_2d(&prm.tm_gu, dtype, gu, 2 * I, M, 2 * I, kEC, kBM, CU_TENSOR_MAP_SWIZZLE_64B)) != MT_OK) return st;
  if ((st = map_2d(&prm.tm_out, dtype, y, I, M, I, kEC, kBM, CU_TENSOR_MAP_SWIZZLE_64B)) != MT_OK) return st;
  return launch<0>(prm, dtype, M, K, 2 * I, static_cast<cudaStream_t>(stream));
}

extern "C" int mt_swiglu_gemm_bwd(const void* dout, const void* w2t, const void* gu, void* dgu, int dtype, int64_t M,
                                  int64_t H, int64_t I, uint32_t* status, void* stream) {
  int st = validate(dtype, M, H, I, {dout, w2t, gu, dgu});
  if (st != MT_OK) return st;
  if (M == 0) return MT_OK;
  if (status == nullptr) return MT_ERR_INVALID_ARGUMENT;
  if ((st = bind_device_of(dout)) != MT_OK) return st;
  if ((st = check_arch()) != MT_OK) return st;
  GemmParams prm;
  prm.status = status;
  if ((st = map_2d(&prm.tm_a, dtype, dout, H, M, H, kBK, kBM, CU_TENSOR_MAP_SWIZZLE_128B)) != MT_OK) return st;
  if ((st = map_2d(&prm.tm_b, dtype, w2t, H, I, H, kBK, b_box_rows(1, M), CU_TENSOR_MAP_SWIZZLE_128B)) != MT_OK)
    return st;
  if ((st = map_2d(&prm.tm_gu, dtype, gu, 2 * I, M, 2 * I, kEC, kBM, CU_TENSOR_MAP_SWIZZLE_64B)) != MT_OK) return st;
  if ((st = map_2d(&prm.tm_out, dtype, dgu, 2 * I, M, 2 * I, kEC, kBM, CU_TENSOR_MAP_SWIZZLE_64B)) != MT_OK) return st;
  return launch<1>(prm, dtype, M, H, I, static_cast<cudaStream_t>(stream));
}

extern "C" int mt_qkv_rope_gemm(const void* x, const void* w, void* qkv, const void* rope_cos, const void* rope_sin,
                                int64_t rope_ld, int dtype, int64_t M, int64_t K, int64_t N, int64_t rot_cols,
                                int64_t seq, int64_t head_dim, uint32_t* status, void* stream) {
  if (dtype != MT_BF16 && dtype != MT_F16) return MT_ERR_UNSUPPORTED_DTYPE;
  if (M < 0 || K <= 0 || N <= 0 || seq <= 0 || rot_cols < 0 || rot_cols > N) return MT_ERR_INVALID_ARGUMENT;
  if (M > 0 && M % seq != 0) return MT_ERR_INVALID_ARGUMENT;  // whole sequences of seq tokens
  if (N % kBN != 0 || K % 8 != 0 || (head_dim != 32 && head_dim != 64) || rot_cols % head_dim != 0)
    return MT_ERR_UNSUPPORTED_LAYOUT;
  if (M > 0x7fffffffLL - kBM || N > 0x7fffffffLL) return MT_ERR_INVALID_ARGUMENT;
  if (M == 0) return MT_OK;
  if (status == nullptr || rope_cos == nullptr || rope_sin == nullptr || rope_ld < head_dim / 2) return MT_ERR_INVALID_ARGUMENT;
  for (const void* q : {x, w, static_cast<const void*>(qkv), rope_cos, rope_sin})
    if (q == nullptr || (reinterpret_cast<uintptr_t>(q) & 15u) != 0) return MT_ERR_UNSUPPORTED_LAYOUT;
  if (rope_ld % 8 != 0) return MT_ERR_UNSUPPORTED_LAYOUT;  // 16-byte table rows (8 pairs per load)
  int st = bind_device_of(x);
  if (st != MT_OK) return st;
  if ((st = check_arch()) != MT_OK) return st;
  GemmParams prm;
  prm.status = status;
  prm.rope_cos = rope_cos;
  prm.rope_sin = rope_sin;
  prm.rope_ld = rope_ld;
  prm.seq = (int)seq;
  prm.head_dim = (int)head_dim;
  prm.rot_cols = (int)rot_cols;
  if ((st = map_2d(&prm.tm_a, dtype, x, K, M, K, kBK, kBM, CU_TENSOR_MAP_SWIZZLE_128B)) != MT_OK) return st;
  if ((st = map_2d(&prm.tm_b, dtype, w, K, N, K, kBK, b_box_rows(2, M), CU_TENSOR_MAP_SWIZZLE_128B)) != MT_OK) return st;
  if ((st = map_2d(&prm.tm_out, dtype, qkv, N, M, N, kEC, kBM, CU_TENSOR_MAP_SWIZZLE_64B)) != MT_OK) return st;
  return launch<2>(prm, dtype, M, K, N, static_cast<cudaStream_t>(stream));
}

