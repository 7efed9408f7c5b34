// Fused linear + cross-entropy for sm_100a.
//
// Reference semantics (duoan/mega-trading):
//   src/mega_trading/kernels/triton_ops.py:64-92 (API, validation), :294-411
//   (chunked Liger-style recipe: logits = H W^T per chunk in HBM, row kernel
//   :822-887 computes loss = (lse - z_y) / n_valid and grad_logits =
//   (softmax - onehot(y)) / n_valid in place, ignored rows contribute 0,
//   all-ignored -> loss 0), torch path :99-112.
//
// B200 design
//   * ce_logits_kernel: a tcgen05 GEMM over tiles of 128 rows x 256 vocab
//     entries (K streamed in 64-wide chunks through a 4-stage TMA ring, 128B
//     swizzle), accumulators double-buffered in TMEM (2 x 256 columns) so the
//     epilogue of one vocab tile overlaps the MMAs of the next.  The epilogue
//     reads the logit tile straight out of TMEM and keeps an online max /
//     sum-exp per row and the target logit; the logits never reach global
//     memory.  The vocabulary is split across CTAs (grid.y) for occupancy;
//     each split writes partial row statistics.
//   * ce_merge_kernel: combines the splits into lse per row and the per-row
//     loss; ce_loss_kernel reduces loss and the valid-row count in one block
//     (fixed order, no host synchronisation).
//   * The backward (dH and dW, logits recomputed on chip) is fused_ce_bwd.cu.
// Warp roles (320 threads): warps 0-7 epilogue in two warpgroups taking
// alternate 32-column steps of a tile (thread = row = TMEM lane; the two
// warpgroups' row statistics are merged at the end), warp 8 TMA producer
// (+ TMEM allocation), warp 9 MMA.
#include <cmath>
#include <type_traits>

#include "common.cuh"

namespace mt {
namespace {

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 64;
constexpr int kThreads = 320;
constexpr int kEC = 32;  // epilogue columns per step
constexpr uint32_t kKernelId = 3;

struct CeCfg {
  static constexpr int NST = 4;
  static constexpr int A_BYTES = kBM * kBK * 2;  // 16 KB
  static constexpr int B_BYTES = kBN * kBK * 2;  // 32 KB
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int OFF_STAGE = 0;
  // [2][128] x {m, s, z} merge area of the two epilogue warpgroups
  static constexpr int OFF_OUT = NST * STAGE;
  static constexpr int OUT_BYTES = 3 * kBM * 4;
  static constexpr int OFF_BAR = OFF_OUT + OUT_BYTES;
  static constexpr int SMEM = OFF_BAR + 256;
};

struct CeParams {
  CUtensorMap tm_h, tm_w;
  const void* labels;
  int labels_i64;
  int64_t ignore_index;
  int N, V, K, n_vtiles, tiles_per_split;
  // outputs: per (row, split) partial max (log2 domain), sum, target logit
  float* part_m;
  float* part_s;
  float* part_z;
  int splits;
  uint32_t* status;
};

__device__ __forceinline__ int64_t load_label(const CeParams& p, int row) {
  return p.labels_i64 ? static_cast<const int64_t*>(p.labels)[row] : (int64_t) static_cast<const int32_t*>(p.labels)[row];
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) ce_logits_kernel(const __grid_constant__ CeParams p) {
  using C = CeCfg;
  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = warp_id();
  const int lane = lane_id();
  if ((smem_u32(smem) & 1023u) != 0) {
    if (threadIdx.x == 0) atomicCAS(p.status, 0u, (kKernelId << 16) | 0xFFFFu);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* full = bars;                  // [NST]
  uint64_t* empty = bars + C::NST;        // [NST]
  uint64_t* acc_full = bars + 2 * C::NST; // [2]
  uint64_t* acc_empty = acc_full + 2;     // [2]
  uint64_t* fin = acc_full + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 24);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 25);

  const int row0 = blockIdx.x * kBM;
  const int split = blockIdx.y;
  const int vt0 = split * p.tiles_per_split;
  const int vt1 = min(vt0 + p.tiles_per_split, p.n_vtiles);
  const int n_vt = max(vt1 - vt0, 0);
  const int n_k = (p.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::NST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&acc_full[s], 1);
      mbar_init(&acc_empty[s], 256);
    }
    mbar_init(fin, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 8) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const WaitCtx wc{p.status, abort_flag, kKernelId};

  if (warp == 8) {
    if (lane == 0) {
      tma_prefetch_desc(&p.tm_h);
      tma_prefetch_desc(&p.tm_w);
      int it = 0;
      bool ok = true;
      for (int vt = vt0; ok && vt < vt1; ++vt) {
        for (int kc = 0; kc < n_k; ++kc, ++it) {
          const int st = it % C::NST;
          if (it >= C::NST && !wait_bounded(wc, &empty[st], ((it / C::NST) & 1) ^ 1, 1)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + C::OFF_STAGE + st * C::STAGE;
          mbar_arrive_expect_tx(&full[st], C::STAGE);
          tma_load_2d(sa, &p.tm_h, &full[st], kc * kBK, row0);
          tma_load_2d(sa + C::A_BYTES, &p.tm_w, &full[st], kc * kBK, vt * kBN);
        }
      }
      if (*abort_flag) {
        for (int j = (it > C::NST ? it - C::NST : 0); j < it; ++j)
          wait_drain(wc, &full[j % C::NST], (j / C::NST) & 1, 11);
      }
    }
  } else if (warp == 9) {
    if (lane == 0) {
      constexpr int kBf16 = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
      constexpr uint32_t idesc = make_idesc(kBM, kBN, kBf16, 0, 0);
      const uint32_t base = smem_u32(smem + C::OFF_STAGE);
      int it = 0;
      bool ok = true;
      for (int t = 0; ok && t < n_vt; ++t) {
        const int buf = t & 1;
        if (t >= 2 && !wait_bounded(wc, &acc_empty[buf], ((t >> 1) & 1) ^ 1, 2)) break;
        tc_fence_after();
        const uint32_t d = tmem + buf * kBN;
        for (int kc = 0; kc < n_k; ++kc, ++it) {
          const int st = it % C::NST;
          if (!wait_bounded(wc, &full[st], (it / C::NST) & 1, 3)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = base + st * C::STAGE;
          const uint32_t b = a + C::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            umma_ss(d, make_sdesc(a + kk * 32, 16, 1024, kSwizzle128), make_sdesc(b + kk * 32, 16, 1024, kSwizzle128),
                    idesc, (kc > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&empty[st]);
        }
        if (ok) umma_commit(&acc_full[buf]);
      }
      umma_commit(fin);
      wait_drain(wc, fin, 0, 13);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int wg = warp >> 2;          // takes the 32-column steps c with c % 2 == wg
    const int r = threadIdx.x & 127;   // row within the tile = TMEM lane
    const int row = row0 + r;
    const bool in_rows = row < p.N;
    const int64_t label = in_rows ? load_label(p, row) : p.ignore_index;
    const bool valid = in_rows && label != p.ignore_index && label >= 0 && label < p.V;
    if (wg == 0 && in_rows && label != p.ignore_index && (label < 0 || label >= p.V))
      atomicCAS(p.status, 0u, (kKernelId << 16) | 0xEEEEu);  // out-of-range target
    const uint32_t lane_off = uint32_t((warp & 3) * 32) << 16;
    constexpr float kLog2e = 1.4426950408889634f;
    float m = -INFINITY, s = 0.f, zy = NAN;
    bool ok = true;
    for (int t = 0; t < n_vt; ++t) {
      const int buf = t & 1;
      const int vbase = (vt0 + t) * kBN;
      if (!__all_sync(0xffffffffu, wait_bounded(wc, &acc_full[buf], (t >> 1) & 1, 8))) {
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll 1
      for (int c = wg; c < kBN / kEC; c += 2) {
        uint32_t z[32];
        tmem_ld32(tmem + lane_off + buf * kBN + c * kEC, z);
        tmem_ld_wait();
        if (c + 2 >= kBN / kEC) {
          tc_fence_before();
          mbar_arrive(&acc_empty[buf]);
        }
        const int col0 = vbase + c * kEC;
        float x[32];
        float cm = -INFINITY;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          x[i] = (col0 + i < p.V) ? __uint_as_float(z[i]) * kLog2e : -INFINITY;
          cm = fmaxf(cm, x[i]);
        }
        const float mn = fmaxf(m, cm);
        float cs = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i) cs += fast_exp2(x[i] - mn);
        s = (m == -INFINITY ? 0.f : s * fast_exp2(m - mn)) + cs;
        m = mn;
        if (valid && label >= col0 && label < col0 + 32) {
          const int li = int(label - col0);
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (i == li) zy = __uint_as_float(z[i]);
        }
      }
    }
    // merge the two warpgroups' running statistics of each row
    float* mg = reinterpret_cast<float*>(smem + C::OFF_OUT);
    if (wg == 1) {
      mg[r] = m;
      mg[128 + r] = s;
      mg[256 + r] = zy;
    }
    named_bar_sync(3, 256);
    if (wg == 0) {
      const float m1 = mg[r], s1 = mg[128 + r], z1 = mg[256 + r];
      const float mn = fmaxf(m, m1);
      const float sm = (m == -INFINITY ? 0.f : s * fast_exp2(m - mn)) + (m1 == -INFINITY ? 0.f : s1 * fast_exp2(m1 - mn));
      const float zm = isnan(zy) ? z1 : zy;
      if (ok && in_rows) {
        const int64_t idx = int64_t(row) * p.splits + split;
        p.part_m[idx] = mn;
        p.part_s[idx] = sm;
        p.part_z[idx] = zm;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Combine split statistics: lse (natural log) and lse2 (log2 domain) per row,
// per-row loss (lse - z_y) for valid rows, 0 otherwise.
__global__ void ce_merge_kernel(const float* __restrict__ pm, const float* __restrict__ ps,
                                const float* __restrict__ pz, int splits, int N, const void* labels, int labels_i64,
                                int64_t ignore_index, int V, float* __restrict__ lse2, float* __restrict__ row_loss,
                                float* __restrict__ row_valid) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= N) return;
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, pm[int64_t(row) * splits + s]);
  float S = 0.f, z = NAN;
  for (int s = 0; s < splits; ++s) {
    const float ms = pm[int64_t(row) * splits + s];
    if (ms != -INFINITY) S += ps[int64_t(row) * splits + s] * exp2f(ms - M);
    const float zs = pz[int64_t(row) * splits + s];
    if (!isnan(zs)) z = zs;
  }
  const float l2 = M + log2f(S);
  lse2[row] = l2;
  const int64_t label = labels_i64 ? static_cast<const int64_t*>(labels)[row]
                                   : (int64_t) static_cast<const int32_t*>(labels)[row];
  const bool valid = label != ignore_index && label >= 0 && label < V;
  row_loss[row] = valid ? (l2 * 0.69314718055994530942f - z) : 0.f;
  row_valid[row] = valid ? 1.f : 0.f;
}

// One block: loss = sum(row_loss) / n_valid (0 if none), scal = {loss, n_valid, inv_n}.
__global__ void __launch_bounds__(1024) ce_loss_kernel(const float* __restrict__ row_loss,
                                                       const float* __restrict__ row_valid, int N,
                                                       float* __restrict__ scal, float* __restrict__ loss_out) {
  __shared__ float sl[32], sv[32];
  float l = 0.f, v = 0.f;
  for (int i = threadIdx.x; i < N; i += blockDim.x) {
    l += row_loss[i];
    v += row_valid[i];
  }
  l = warp_sum(l);
  v = warp_sum(v);
  if (lane_id() == 0) {
    sl[warp_id()] = l;
    sv[warp_id()] = v;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int nw = (blockDim.x + 31) / 32;
    l = threadIdx.x < nw ? sl[threadIdx.x] : 0.f;
    v = threadIdx.x < nw ? sv[threadIdx.x] : 0.f;
    l = warp_sum(l);
    v = warp_sum(v);
    if (threadIdx.x == 0) {
      const float inv = v > 0.f ? 1.f / v : 0.f;
      const float loss = l * inv;
      scal[0] = loss;
      scal[1] = v;
      scal[2] = inv;
      loss_out[0] = loss;
    }
  }
}

struct CeWorkspace {
  float *pm, *ps, *pz, *lse2, *row_loss, *row_valid, *scal;
  int64_t bytes;
};

CeWorkspace ce_carve(void* base, int64_t N, int splits) {
  auto up = [](int64_t x) { return (x + 255) / 256 * 256; };
  char* p = static_cast<char*>(base);
  CeWorkspace w;
  const int64_t a = up(N * splits * 4), b = up(N * 4);
  w.pm = reinterpret_cast<float*>(p);
  w.ps = reinterpret_cast<float*>(p + a);
  w.pz = reinterpret_cast<float*>(p + 2 * a);
  w.lse2 = reinterpret_cast<float*>(p + 3 * a);
  w.row_loss = reinterpret_cast<float*>(p + 3 * a + b);
  w.row_valid = reinterpret_cast<float*>(p + 3 * a + 2 * b);
  w.scal = reinterpret_cast<float*>(p + 3 * a + 3 * b);
  w.bytes = 3 * a + 3 * b + 256;
  return w;
}

int ce_splits(int64_t N, int64_t V) {
  const int64_t row_tiles = (N + kBM - 1) / kBM;
  const int64_t vt = (V + kBN - 1) / kBN;
  const int64_t sms = get_sm_count();
  // enough CTAs for ~4 waves, never more splits than vocab tiles
  int64_t s = (4 * sms + row_tiles - 1) / row_tiles;
  if (s < 1) s = 1;
  if (s > vt) s = vt;
  if (s > 16) s = 16;
  return (int)s;
}

int ce_maps(CeParams& prm, const void* hidden, const void* weight, int dtype, int64_t N, int64_t V, int64_t K) {
  const CUtensorMapDataType dt = dtype == MT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  uint64_t dims_h[2] = {(uint64_t)K, (uint64_t)N};
  uint64_t str_h[1] = {(uint64_t)K * 2};
  uint32_t box_h[2] = {kBK, kBM};
  int st = encode_tensor_map(&prm.tm_h, dt, 2, const_cast<void*>(hidden), dims_h, str_h, box_h,
                             CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != MT_OK) return st;
  uint64_t dims_w[2] = {(uint64_t)K, (uint64_t)V};
  uint32_t box_w[2] = {kBK, kBN};
  return encode_tensor_map(&prm.tm_w, dt, 2, const_cast<void*>(weight), dims_w, str_h, box_w,
                           CU_TENSOR_MAP_SWIZZLE_128B);
}

int ce_validate(const void* hidden, const void* weight, const void* labels, int dtype, int64_t N, int64_t V, int64_t K) {
  if (dtype != MT_BF16 && dtype != MT_F16) return MT_ERR_UNSUPPORTED_DTYPE;
  if (N < 0 || V <= 0 || K <= 0) return MT_ERR_INVALID_ARGUMENT;
  if (N > 0x7fffffffLL - kBM || V > 0x7fffffffLL) return MT_ERR_INVALID_ARGUMENT;
  if (N > 0 && (hidden == nullptr || weight == nullptr || labels == nullptr)) return MT_ERR_INVALID_ARGUMENT;
  if (K % 8 != 0) return MT_ERR_UNSUPPORTED_LAYOUT;
  if ((reinterpret_cast<uintptr_t>(hidden) & 15u) || (reinterpret_cast<uintptr_t>(weight) & 15u))
    return MT_ERR_UNSUPPORTED_LAYOUT;
  return MT_OK;
}

template <typename T>
int launch_logits(const CeParams& prm, int64_t N, cudaStream_t stream) {
  using C = CeCfg;
  auto kern = ce_logits_kernel<T>;
  int st = set_smem_limit((const void*)kern, C::SMEM);
  if (st != MT_OK) return st;
  dim3 grid((unsigned)((N + kBM - 1) / kBM), (unsigned)prm.splits);
  kern<<<grid, kThreads, C::SMEM, stream>>>(prm);
  return check_launch("fused_ce_lse");
}

}  // namespace
}  // namespace mt

using namespace mt;

extern "C" int64_t mt_fused_ce_workspace_bytes(int64_t N, int64_t V) {
  if (N <= 0 || V <= 0) return 256;
  return ce_carve(nullptr, N, ce_splits(N, V)).bytes;
}

extern "C" int mt_fused_ce_fwd(const void* hidden, const void* weight, const void* labels, int labels_i64,
                               int64_t ignore_index, int dtype, int64_t N, int64_t V, int64_t K, float* loss,
                               float* lse2_out, void* workspace, int64_t workspace_bytes, uint32_t* status,
                               void* stream) {
  int st = ce_validate(hidden, weight, labels, dtype, N, V, K);
  if (st != MT_OK) return st;
  if (loss == nullptr || status == nullptr || workspace == nullptr) return MT_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return MT_ERR_WORKSPACE;
  auto s = static_cast<cudaStream_t>(stream);
  const int splits = N > 0 ? ce_splits(N, V) : 1;
  CeWorkspace ws = ce_carve(workspace, N, splits);
  if (workspace_bytes < ws.bytes) return MT_ERR_WORKSPACE;
  if (N == 0) {
    cudaError_t e = cudaMemsetAsync(loss, 0, 4, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(ws.scal, 0, 16, s);
    return e == cudaSuccess ? MT_OK : MT_ERR_LAUNCH;
  }
  if ((st = bind_device_of(hidden)) != MT_OK) return st;
  if ((st = check_arch()) != MT_OK) return st;
  CeParams prm;
  if ((st = ce_maps(prm, hidden, weight, dtype, N, V, K)) != MT_OK) return st;
  prm.labels = labels;
  prm.labels_i64 = labels_i64;
  prm.ignore_index = ignore_index;
  prm.N = (int)N;
  prm.V = (int)V;
  prm.K = (int)K;
  prm.n_vtiles = (int)((V + kBN - 1) / kBN);
  prm.splits = splits;
  prm.tiles_per_split = (prm.n_vtiles + splits - 1) / splits;
  prm.part_m = ws.pm;
  prm.part_s = ws.ps;
  prm.part_z = ws.pz;
  prm.status = status;
  st = dtype == MT_BF16 ? launch_logits<__nv_bfloat16>(prm, N, s) : launch_logits<__half>(prm, N, s);
  if (st != MT_OK) return st;
  ce_merge_kernel<<<(unsigned)((N + 255) / 256), 256, 0, s>>>(ws.pm, ws.ps, ws.pz, splits, (int)N, labels, labels_i64,
                                                               ignore_index, (int)V, ws.lse2, ws.row_loss,
                                                               ws.row_valid);
  if ((st = check_launch("fused_ce_merge")) != MT_OK) return st;
  ce_loss_kernel<<<1, 1024, 0, s>>>(ws.row_loss, ws.row_valid, (int)N, ws.scal, loss);
  if ((st = check_launch("fused_ce_loss")) != MT_OK) return st;
  if (lse2_out != nullptr) {
    cudaError_t e = cudaMemcpyAsync(lse2_out, ws.lse2, N * 4, cudaMemcpyDeviceToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(lse2_out + N, ws.scal, 12, cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) {
      set_last_error("cudaMemcpyAsync(lse2)", e);
      return MT_ERR_LAUNCH;
    }
  }
  return MT_OK;
}
