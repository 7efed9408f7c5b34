// RMSNorm and fused residual-add + RMSNorm, forward and backward.
//
// Reference semantics (duoan/mega-trading):
//   forward  src/mega_trading/kernels/triton_ops.py:528-538 (RMSNorm),
//            :541-566 (add+RMSNorm); torch path F.rms_norm (model.py:269)
//   backward :633-665 and :569-608, dW finished by a torch sum (:183, :287)
//
// B200 design: one warp per row, 16-byte vector loads (8 elements per lane
// per chunk), the row held in registers between the reduction and the
// normalisation, warp-shuffle reductions, fp32 math for every dtype.  The
// backward keeps per-lane dW partials in registers across the rows a warp
// visits, reduces the 8 warps of a block through shared memory and writes one
// fp32 partial row per block into the caller's workspace; a second small
// kernel sums the partials in a fixed order (deterministic dW).
#include <mutex>

#include "common.cuh"

namespace mt {
namespace {

constexpr int kWarps = 8;           // rows in flight per block
constexpr int kChunk = 8;           // elements per lane per chunk
constexpr int kBwdBlocksPerSM = 3;  // persistent backward grid: at most 3 resident blocks per SM

// Load / store 8 consecutive elements as floats (16 or 32 bytes).
template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]) {
  if constexpr (sizeof(T) == 2) {
    load_vec<T, 8>(p, v);
  } else {
    float a[4], b[4];
    load_vec<T, 4>(p, a);
    load_vec<T, 4>(p + 4, b);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[i] = a[i];
      v[i + 4] = b[i];
    }
  }
}
template <typename T>
__device__ __forceinline__ void store8(T* p, const float (&v)[8]) {
  if constexpr (sizeof(T) == 2) {
    store_vec<T, 8>(p, v);
  } else {
    float a[4], b[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      a[i] = v[i];
      b[i] = v[i + 4];
    }
    store_vec<T, 4>(p, a);
    store_vec<T, 4>(p + 4, b);
  }
}

// ---------------------------------------------------------------------------
// forward: vectorised, row in registers (NC chunks of 8 per lane)
//   ADD: s = round_to<TR>(x + r) is stored as new_residual and normalised.
// ---------------------------------------------------------------------------
template <typename TX, typename TW, typename TY, typename TR, bool ADD, int NC>
__global__ void __launch_bounds__(kWarps * 32) rms_fwd_vec(const TX* __restrict__ x, const TR* __restrict__ r,
                                                           const TW* __restrict__ w, TR* __restrict__ new_res,
                                                           TY* __restrict__ y, float* __restrict__ rstd,
                                                           int64_t rows, int dim, float eps) {
  const int lane = lane_id();
  const int64_t row = int64_t(blockIdx.x) * kWarps + warp_id();
  if (row >= rows) return;
  const TX* xr = x + row * dim;
  float v[NC][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int col = (c * 32 + lane) * kChunk;
    if (col < dim) {
      load8<TX>(xr + col, v[c]);
      if constexpr (ADD) {
        float rv[8];
        load8<TR>(r + row * dim + col, rv);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[c][i] = round_to<TR>(v[c][i] + rv[i]);
        store8<TR>(new_res + row * dim + col, v[c]);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) ss = fmaf(v[c][i], v[c][i], ss);
    }
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / float(dim) + eps);
  if (lane == 0) rstd[row] = inv;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int col = (c * 32 + lane) * kChunk;
    if (col < dim) {
      float wv[8], o[8];
      load8<TW>(w + col, wv);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = v[c][i] * inv * wv[i];
      store8<TY>(y + row * dim + col, o);
    }
  }
}

// Generic forward (any dim / alignment): one warp per row, scalar accesses,
// two passes over the row.
template <typename TX, typename TW, typename TY, typename TR, bool ADD>
__global__ void __launch_bounds__(kWarps * 32) rms_fwd_scalar(const TX* __restrict__ x, const TR* __restrict__ r,
                                                              const TW* __restrict__ w, TR* __restrict__ new_res,
                                                              TY* __restrict__ y, float* __restrict__ rstd,
                                                              int64_t rows, int dim, float eps) {
  const int lane = lane_id();
  const int64_t row = int64_t(blockIdx.x) * kWarps + warp_id();
  if (row >= rows) return;
  float ss = 0.f;
  for (int col = lane; col < dim; col += 32) {
    float s = to_f32<TX>(x[row * dim + col]);
    if constexpr (ADD) {
      s = round_to<TR>(s + to_f32<TR>(r[row * dim + col]));
      new_res[row * dim + col] = from_f32<TR>(s);
    }
    ss = fmaf(s, s, ss);
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / float(dim) + eps);
  if (lane == 0) rstd[row] = inv;
  for (int col = lane; col < dim; col += 32) {
    float s = to_f32<TX>(x[row * dim + col]);
    if constexpr (ADD) s = round_to<TR>(s + to_f32<TR>(r[row * dim + col]));
    y[row * dim + col] = from_f32<TY>(s * inv * to_f32<TW>(w[col]));
  }
}

// ---------------------------------------------------------------------------
// backward: persistent grid, warps stride over rows.
//   dn   = dy * w
//   dx   = rstd * (dn - x * rstd^2 * sum(dn * x) / dim)  (+ g_res if GRES)
//   dw_p = sum_rows dy * x * rstd                       (per block partial)
// Each warp holds its current row (x, dy and g_res as raw 16-byte words) in
// registers and issues the loads of its next row before it reduces and writes
// the current one, so two rows per warp are in flight and the per-row
// shuffle reduction hides under the next row's load latency.  The dW
// partials stay in registers across all rows the warp visits.
// ---------------------------------------------------------------------------
template <typename T>
struct Raw8 {  // 8 consecutive elements as raw 16-byte words
  uint4 q[sizeof(T) / 2];
};

template <typename T>
__device__ __forceinline__ void raw_load(Raw8<T>& r, const T* p) {
  const uint4* s = reinterpret_cast<const uint4*>(p);
#pragma unroll
  for (int i = 0; i < int(sizeof(T) / 2); ++i) r.q[i] = __ldg(s + i);
}

template <typename T>
__device__ __forceinline__ void raw_unpack(const Raw8<T>& r, float (&v)[8]) {
  if constexpr (sizeof(T) == 4) {
    const uint32_t* u = reinterpret_cast<const uint32_t*>(r.q);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(u[i]);
  } else {
    const uint32_t* u = reinterpret_cast<const uint32_t*>(r.q);
#pragma unroll
    for (int i = 0; i < 4; ++i) unpack2<T>(u[i], v[2 * i], v[2 * i + 1]);
  }
}

// Sum the 8 warps' dW partials of a block through shared memory and write the
// block's partial row.
template <int NC>
__device__ __forceinline__ void block_partial(const float (&acc)[NC][8], float* red, float* __restrict__ partial,
                                              int dim) {
  const int lane = lane_id();
  const int warp = warp_id();
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int col = (c * 32 + lane) * kChunk;
    if (col < dim) {
#pragma unroll
      for (int i = 0; i < 8; ++i) red[warp * dim + col + i] = acc[c][i];
    }
  }
  __syncthreads();
  for (int col = threadIdx.x; col < dim; col += blockDim.x) {
    float s = 0.f;
#pragma unroll
    for (int q = 0; q < kWarps; ++q) s += red[q * dim + col];
    partial[int64_t(blockIdx.x) * dim + col] = s;
  }
}

// Rows wider than 1024 elements (6 or 8 chunks per lane): only the dW partials
// stay in registers; each row is read twice (dot product, then dx), the second
// time from L1.
template <typename TX, typename TW, typename TG, typename TGR, typename TD, bool GRES, int NC>
__global__ void __launch_bounds__(kWarps * 32, 1)
    rms_bwd_reread(const TX* __restrict__ x, const TW* __restrict__ w, const float* __restrict__ rstd,
                   const TG* __restrict__ dy, const TGR* __restrict__ gres, TD* __restrict__ dx,
                   TG* __restrict__ dx2, float* __restrict__ partial, int64_t rows, int dim) {
  extern __shared__ float red[];  // [kWarps][dim]
  const int lane = lane_id();
  const int warp = warp_id();
  float acc[NC][8];
#pragma unroll
  for (int c = 0; c < NC; ++c)
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[c][i] = 0.f;
  for (int64_t row = int64_t(blockIdx.x) * kWarps + warp; row < rows; row += int64_t(gridDim.x) * kWarps) {
    const float inv = rstd[row];
    const TX* xr = x + row * dim;
    const TG* gr_ = dy + row * dim;
    float dot = 0.f;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int col = (c * 32 + lane) * kChunk;
      if (col < dim) {
        float xv[8], gv[8], wv[8];
        load8<TX>(xr + col, xv);
        load8<TG>(gr_ + col, gv);
        load8<TW>(w + col, wv);
#pragma unroll
        for (int i = 0; i < 8; ++i) dot = fmaf(gv[i] * wv[i], xv[i], dot);
      }
    }
    dot = warp_sum(dot);
    const float k = inv * inv * dot / float(dim);
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int col = (c * 32 + lane) * kChunk;
      if (col < dim) {
        float xv[8], gv[8], wv[8], o[8];
        load8<TX>(xr + col, xv);
        load8<TG>(gr_ + col, gv);
        load8<TW>(w + col, wv);
        float rg[8];
        if constexpr (GRES) load8<TGR>(gres + row * dim + col, rg);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          o[i] = inv * (gv[i] * wv[i] - xv[i] * k);
          if constexpr (GRES) o[i] += rg[i];
          acc[c][i] = fmaf(gv[i], xv[i] * inv, acc[c][i]);
        }
        store8<TD>(dx + row * dim + col, o);
        if (dx2 != nullptr) store8<TG>(dx2 + row * dim + col, o);
      }
    }
  }
  block_partial<NC>(acc, red, partial, dim);
}

// Rows of at most 1024 elements (1 to 4 chunks per lane): row in registers,
// next row prefetched.
template <typename TX, typename TW, typename TG, typename TGR, typename TD, bool GRES, int NC>
__global__ void __launch_bounds__(kWarps * 32)
    rms_bwd_vec(const TX* __restrict__ x, const TW* __restrict__ w, const float* __restrict__ rstd,
                const TG* __restrict__ dy, const TGR* __restrict__ gres, TD* __restrict__ dx,
                TG* __restrict__ dx2, float* __restrict__ partial, int64_t rows, int dim) {
  // dx2 (optional): dx once more, rounded to dy's dtype
  extern __shared__ float red[];  // [kWarps][dim]
  const int lane = lane_id();
  const int warp = warp_id();
  const int64_t stride = int64_t(gridDim.x) * kWarps;
  float acc[NC][8];
#pragma unroll
  for (int c = 0; c < NC; ++c)
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[c][i] = 0.f;

  Raw8<TX> xc[NC];
  Raw8<TG> gc[NC];
  Raw8<TGR> rc[GRES ? NC : 1];
  float inv_c = 0.f;
  auto load_row = [&](int64_t row, Raw8<TX>(&xs)[NC], Raw8<TG>(&gs)[NC], Raw8<TGR>(&rs)[GRES ? NC : 1],
                      float& inv) {
    inv = __ldg(rstd + row);
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int col = (c * 32 + lane) * kChunk;
      if (col < dim) {
        raw_load<TX>(xs[c], x + row * dim + col);
        raw_load<TG>(gs[c], dy + row * dim + col);
        if constexpr (GRES) raw_load<TGR>(rs[c], gres + row * dim + col);
      }
    }
  };

  int64_t row = int64_t(blockIdx.x) * kWarps + warp;
  if (row < rows) load_row(row, xc, gc, rc, inv_c);
  for (; row < rows; row += stride) {
    Raw8<TX> xn[NC];
    Raw8<TG> gn[NC];
    Raw8<TGR> rn[GRES ? NC : 1];
    float inv_n = 0.f;
    if (row + stride < rows) load_row(row + stride, xn, gn, rn, inv_n);

    float dot = 0.f;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int col = (c * 32 + lane) * kChunk;
      if (col < dim) {
        float xv[8], gv[8], wv[8];
        raw_unpack<TX>(xc[c], xv);
        raw_unpack<TG>(gc[c], gv);
        load8<TW>(w + col, wv);
#pragma unroll
        for (int i = 0; i < 8; ++i) dot = fmaf(gv[i] * wv[i], xv[i], dot);
      }
    }
    dot = warp_sum(dot);
    const float inv = inv_c;
    const float k = inv * inv * dot / float(dim);
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int col = (c * 32 + lane) * kChunk;
      if (col < dim) {
        float xv[8], gv[8], wv[8], o[8];
        raw_unpack<TX>(xc[c], xv);
        raw_unpack<TG>(gc[c], gv);
        load8<TW>(w + col, wv);
        float rg[8];
        if constexpr (GRES) raw_unpack<TGR>(rc[c], rg);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          o[i] = inv * (gv[i] * wv[i] - xv[i] * k);
          if constexpr (GRES) o[i] += rg[i];
          acc[c][i] = fmaf(gv[i], xv[i] * inv, acc[c][i]);
        }
        store8<TD>(dx + row * dim + col, o);
        if (dx2 != nullptr) store8<TG>(dx2 + row * dim + col, o);
      }
    }
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      xc[c] = xn[c];
      gc[c] = gn[c];
      if constexpr (GRES) rc[c] = rn[c];
    }
    inv_c = inv_n;
  }
  block_partial<NC>(acc, red, partial, dim);
}

template <typename TX, typename TW, typename TG, typename TGR, typename TD, bool GRES>
__global__ void __launch_bounds__(kWarps * 32) rms_bwd_scalar(const TX* __restrict__ x, const TW* __restrict__ w,
                                                              const float* __restrict__ rstd,
                                                              const TG* __restrict__ dy, const TGR* __restrict__ gres,
                                                              TD* __restrict__ dx, TG* __restrict__ dx2,
                                                              float* __restrict__ partial, int64_t rows, int dim) {
  // dW partial per block: thread t owns columns t, t + blockDim, ... and
  // loops over the block's rows itself (no cross-warp reduction needed).
  for (int col = threadIdx.x; col < dim; col += blockDim.x) {
    float s = 0.f;
    for (int64_t row = blockIdx.x; row < rows; row += gridDim.x)
      s += to_f32<TG>(dy[row * dim + col]) * to_f32<TX>(x[row * dim + col]) * rstd[row];
    partial[int64_t(blockIdx.x) * dim + col] = s;
  }
  const int lane = lane_id();
  for (int64_t row = int64_t(blockIdx.x) * kWarps + warp_id(); row < rows; row += int64_t(gridDim.x) * kWarps) {
    const float inv = rstd[row];
    float dot = 0.f;
    for (int col = lane; col < dim; col += 32)
      dot += to_f32<TG>(dy[row * dim + col]) * to_f32<TW>(w[col]) * to_f32<TX>(x[row * dim + col]);
    dot = warp_sum(dot);
    const float k = inv * inv * dot / float(dim);
    for (int col = lane; col < dim; col += 32) {
      float o = inv * (to_f32<TG>(dy[row * dim + col]) * to_f32<TW>(w[col]) - to_f32<TX>(x[row * dim + col]) * k);
      if constexpr (GRES) o += to_f32<TGR>(gres[row * dim + col]);
      dx[row * dim + col] = from_f32<TD>(o);
      if (dx2 != nullptr) dx2[row * dim + col] = from_f32<TG>(o);
    }
  }
}

// Second stage: dw[col] = sum over blocks of partial[block][col], in a fixed
// order (32 row-lanes per column, then a tree over the lanes).
template <typename TW>
__global__ void __launch_bounds__(1024) dw_reduce(const float* __restrict__ partial, int nblocks, int dim,
                                                  TW* __restrict__ dw) {
  __shared__ float s[32][33];
  const int col = blockIdx.x * 32 + threadIdx.x;
  float v = 0.f;
  if (col < dim)
    for (int b = threadIdx.y; b < nblocks; b += 32) v += partial[int64_t(b) * dim + col];
  s[threadIdx.y][threadIdx.x] = v;
  __syncthreads();
  if (threadIdx.y == 0) {
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) t += s[i][threadIdx.x];
    if (col < dim) dw[col] = from_f32<TW>(t);
  }
}

// ---------------------------------------------------------------------------
// dispatch helpers
// ---------------------------------------------------------------------------
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <typename F>
int with_dtype(int code, F&& f) {
  switch (code) {
    case MT_F32: return f(float{});
    case MT_F16: return f(__half{});
    case MT_BF16: return f(__nv_bfloat16{});
    default: return MT_ERR_UNSUPPORTED_DTYPE;
  }
}

int chunks_for(int64_t dim) {
  const int64_t per_lane = (dim + 32 * kChunk - 1) / (32 * kChunk);
  if (per_lane <= 4) return (int)per_lane;  // 1, 2, 3, 4
  if (per_lane <= 6) return 6;
  if (per_lane <= 8) return 8;
  return 0;  // too wide for the register-resident path
}

template <bool ADD, typename TX, typename TW, typename TY, typename TR>
int launch_fwd(const void* x, const void* r, const void* w, void* new_res, void* y, float* rstd, int64_t rows,
               int64_t dim, float eps, cudaStream_t stream) {
  const int nc = chunks_for(dim);
  const bool vec = nc > 0 && dim % kChunk == 0 && aligned16(x) && aligned16(w) && aligned16(y) &&
                   (!ADD || (aligned16(r) && aligned16(new_res)));
  const dim3 grid((unsigned)((rows + kWarps - 1) / kWarps));
  const dim3 block(kWarps * 32);
  auto X = static_cast<const TX*>(x);
  auto R = static_cast<const TR*>(r);
  auto W = static_cast<const TW*>(w);
  auto NR = static_cast<TR*>(new_res);
  auto Y = static_cast<TY*>(y);
  const int d = (int)dim;
  if (vec) {
    switch (nc) {
      case 1: rms_fwd_vec<TX, TW, TY, TR, ADD, 1><<<grid, block, 0, stream>>>(X, R, W, NR, Y, rstd, rows, d, eps); break;
      case 2: rms_fwd_vec<TX, TW, TY, TR, ADD, 2><<<grid, block, 0, stream>>>(X, R, W, NR, Y, rstd, rows, d, eps); break;
      case 3: rms_fwd_vec<TX, TW, TY, TR, ADD, 3><<<grid, block, 0, stream>>>(X, R, W, NR, Y, rstd, rows, d, eps); break;
      case 4: rms_fwd_vec<TX, TW, TY, TR, ADD, 4><<<grid, block, 0, stream>>>(X, R, W, NR, Y, rstd, rows, d, eps); break;
      case 6: rms_fwd_vec<TX, TW, TY, TR, ADD, 6><<<grid, block, 0, stream>>>(X, R, W, NR, Y, rstd, rows, d, eps); break;
      default: rms_fwd_vec<TX, TW, TY, TR, ADD, 8><<<grid, block, 0, stream>>>(X, R, W, NR, Y, rstd, rows, d, eps); break;
    }
  } else {
    rms_fwd_scalar<TX, TW, TY, TR, ADD><<<grid, block, 0, stream>>>(X, R, W, NR, Y, rstd, rows, d, eps);
  }
  return check_launch(ADD ? "add_rms_norm_fwd" : "rms_norm_fwd");
}

int bwd_blocks(int64_t rows) {
  int64_t g = int64_t(get_sm_count()) * kBwdBlocksPerSM;
  const int64_t need = (rows + kWarps - 1) / kWarps;
  if (g > need) g = need;
  return (int)(g < 1 ? 1 : g);
}

template <bool GRES, typename TX, typename TW, typename TG, typename TGR, typename TD, typename TDW>
int launch_bwd(const void* x, const void* w, const float* rstd, const void* dy, const void* gres, void* dx, void* dw,
               void* workspace, int64_t ws_bytes, int64_t rows, int64_t dim, cudaStream_t stream,
               int max_blocks = 0, void* dx2 = nullptr) {
  int nblocks = bwd_blocks(rows);
  if (max_blocks > 0 && nblocks > max_blocks) nblocks = max_blocks;
  if (workspace == nullptr || ws_bytes < int64_t(nblocks) * dim * 4) return MT_ERR_WORKSPACE;
  float* partial = static_cast<float*>(workspace);
  const int nc = chunks_for(dim);
  const bool vec = nc > 0 && dim % kChunk == 0 && aligned16(x) && aligned16(w) && aligned16(dy) && aligned16(dx) &&
                   (!GRES || aligned16(gres)) && (dx2 == nullptr || aligned16(dx2));
  auto X = static_cast<const TX*>(x);
  auto W = static_cast<const TW*>(w);
  auto G = static_cast<const TG*>(dy);
  auto GR = static_cast<const TGR*>(gres);
  auto DX = static_cast<TD*>(dx);
  auto DX2 = static_cast<TG*>(dx2);
  const int d = (int)dim;
  const int smem = kWarps * d * 4;
  if (vec) {
    const void* fn = nullptr;
    switch (nc) {
      case 1: fn = (const void*)rms_bwd_vec<TX, TW, TG, TGR, TD, GRES, 1>; break;
      case 2: fn = (const void*)rms_bwd_vec<TX, TW, TG, TGR, TD, GRES, 2>; break;
      case 3: fn = (const void*)rms_bwd_vec<TX, TW, TG, TGR, TD, GRES, 3>; break;
      case 4: fn = (const void*)rms_bwd_vec<TX, TW, TG, TGR, TD, GRES, 4>; break;
      case 6: fn = (const void*)rms_bwd_reread<TX, TW, TG, TGR, TD, GRES, 6>; break;
      default: fn = (const void*)rms_bwd_reread<TX, TW, TG, TGR, TD, GRES, 8>; break;
    }
    int st = set_smem_limit(fn, smem);
    if (st != MT_OK) return st;
    // one wave: as many blocks as are resident at once (the workspace holds 3 per SM)
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kWarps * 32, smem) == cudaSuccess && per_sm > 0 &&
        per_sm < kBwdBlocksPerSM) {
      const int cap = get_sm_count() * per_sm;
      if (nblocks > cap) nblocks = cap;
    }
    switch (nc) {
      case 1: rms_bwd_vec<TX, TW, TG, TGR, TD, GRES, 1><<<nblocks, kWarps * 32, smem, stream>>>(X, W, rstd, G, GR, DX, DX2, partial, rows, d); break;
      case 2: rms_bwd_vec<TX, TW, TG, TGR, TD, GRES, 2><<<nblocks, kWarps * 32, smem, stream>>>(X, W, rstd, G, GR, DX, DX2, partial, rows, d); break;
      case 3: rms_bwd_vec<TX, TW, TG, TGR, TD, GRES, 3><<<nblocks, kWarps * 32, smem, stream>>>(X, W, rstd, G, GR, DX, DX2, partial, rows, d); break;
      case 4: rms_bwd_vec<TX, TW, TG, TGR, TD, GRES, 4><<<nblocks, kWarps * 32, smem, stream>>>(X, W, rstd, G, GR, DX, DX2, partial, rows, d); break;
      case 6: rms_bwd_reread<TX, TW, TG, TGR, TD, GRES, 6><<<nblocks, kWarps * 32, smem, stream>>>(X, W, rstd, G, GR, DX, DX2, partial, rows, d); break;
      default: rms_bwd_reread<TX, TW, TG, TGR, TD, GRES, 8><<<nblocks, kWarps * 32, smem, stream>>>(X, W, rstd, G, GR, DX, DX2, partial, rows, d); break;
    }
  } else {
    rms_bwd_scalar<TX, TW, TG, TGR, TD, GRES><<<nblocks, kWarps * 32, 0, stream>>>(X, W, rstd, G, GR, DX, DX2, partial, rows, d);
  }
  int st = check_launch(GRES ? "add_rms_norm_bwd" : "rms_norm_bwd");
  if (st != MT_OK) return st;
  dw_reduce<TDW><<<(d + 31) / 32, dim3(32, 32), 0, stream>>>(partial, nblocks, d, static_cast<TDW*>(dw));
  return check_launch("rms_norm_dw_reduce");
}

int validate_rows(const void* a, const void* b, int64_t rows, int64_t dim) {
  if (rows < 0 || dim <= 0 || dim > (1 << 20)) return MT_ERR_INVALID_ARGUMENT;
  if (rows > 0 && (a == nullptr || b == nullptr)) return MT_ERR_INVALID_ARGUMENT;
  return MT_OK;
}

// Supported dtype combinations (x, w, y[, residual]): the all-same-dtype
// cases of the reference API plus the mixed cases of the B200 training step
// (fp32 residual stream, fp32 weights, bf16 normalised output).
#define MT_DT(a) ((a) & 3)
constexpr int key3(int a, int b, int c) { return (a << 4) | (b << 2) | c; }
constexpr int key5(int a, int b, int c, int d, int e) { return (a << 8) | (b << 6) | (c << 4) | (d << 2) | e; }

}  // namespace
}  // namespace mt

using namespace mt;

extern "C" {

int mt_rms_norm_fwd(const void* x, int x_dtype, const void* w, int w_dtype, void* y, int y_dtype, float* rstd,
                    int64_t rows, int64_t dim, float eps, void* stream) {
  int st = validate_rows(x, y, rows, dim);
  if (st != MT_OK) return st;
  if (rows == 0) return MT_OK;
  auto s = static_cast<cudaStream_t>(stream);
  using bf = __nv_bfloat16;
  using hf = __half;
  switch (key3(x_dtype, w_dtype, y_dtype)) {
#define CASE(a, b, c, TA, TB, TC) \
  case key3(a, b, c): return launch_fwd<false, TA, TB, TC, TA>(x, nullptr, w, nullptr, y, rstd, rows, dim, eps, s);
    CASE(MT_BF16, MT_BF16, MT_BF16, bf, bf, bf)
    CASE(MT_F16, MT_F16, MT_F16, hf, hf, hf)
    CASE(MT_F32, MT_F32, MT_F32, float, float, float)
    CASE(MT_BF16, MT_F32, MT_BF16, bf, float, bf)
    CASE(MT_F16, MT_F32, MT_F16, hf, float, hf)
    CASE(MT_F32, MT_F32, MT_BF16, float, float, bf)
#undef CASE
    default: return MT_ERR_UNSUPPORTED_DTYPE;
  }
}

int64_t mt_rms_norm_bwd_workspace_bytes(int64_t rows, int64_t dim) {
  return int64_t(bwd_blocks(rows)) * dim * 4;
}

static int zero_dw(void* dw, int dw_dtype, int64_t dim, cudaStream_t s) {
  const int64_t esize = dw_dtype == MT_F32 ? 4 : 2;
  cudaError_t e = cudaMemsetAsync(dw, 0, dim * esize, s);
  return e == cudaSuccess ? MT_OK : MT_ERR_LAUNCH;
}

int mt_rms_norm_bwd(const void* x, int x_dtype, const void* w, int w_dtype, const float* rstd, const void* dy,
                    int dy_dtype, void* dx, int dx_dtype, void* dw, int dw_dtype, void* workspace,
                    int64_t workspace_bytes, int64_t rows, int64_t dim, void* stream) {
  int st = validate_rows(x, dx, rows, dim);
  if (st != MT_OK) return st;
  auto s = static_cast<cudaStream_t>(stream);
  if (rows == 0) return zero_dw(dw, dw_dtype, dim, s);
  using bf = __nv_bfloat16;
  using hf = __half;
  switch (key5(x_dtype, w_dtype, dy_dtype, dx_dtype, dw_dtype)) {
#define CASE(a, b, c, d, e, TA, TB, TC, TD, TE)                                                               \
  case key5(a, b, c, d, e):                                                                                    \
    return launch_bwd<false, TA, TB, TC, TC, TD, TE>(x, w, rstd, dy, nullptr, dx, dw, workspace, workspace_bytes, \
                                                 rows, dim, s);
    CASE(MT_BF16, MT_BF16, MT_BF16, MT_BF16, MT_BF16, bf, bf, bf, bf, bf)
    CASE(MT_F16, MT_F16, MT_F16, MT_F16, MT_F16, hf, hf, hf, hf, hf)
    CASE(MT_F32, MT_F32, MT_F32, MT_F32, MT_F32, float, float, float, float, float)
    CASE(MT_BF16, MT_F32, MT_BF16, MT_BF16, MT_F32, bf, float, bf, bf, float)
    CASE(MT_F16, MT_F32, MT_F16, MT_F16, MT_F32, hf, float, hf, hf, float)
    CASE(MT_F32, MT_F32, MT_BF16, MT_F32, MT_F32, float, float, bf, float, float)
#undef CASE
    default: return MT_ERR_UNSUPPORTED_DTYPE;
  }
}

int mt_add_rms_norm_fwd(const void* hidden, const void* residual, int act_dtype, const void* w, int w_dtype,
                        void* new_residual, int res_dtype, void* normed, int normed_dtype, float* rstd, int64_t rows,
                        int64_t dim, float eps, void* stream) {
  int st = validate_rows(hidden, normed, rows, dim);
  if (st != MT_OK) return st;
  if (rows > 0 && (residual == nullptr || new_residual == nullptr)) return MT_ERR_INVALID_ARGUMENT;
  if (rows == 0) return MT_OK;
  auto s = static_cast<cudaStream_t>(stream);
  using bf = __nv_bfloat16;
  using hf = __half;
  // residual input and new residual share res_dtype; hidden may be narrower
  // (the model adds a bf16 branch output into its fp32 residual stream)
  switch (key3(act_dtype, w_dtype, normed_dtype) | (res_dtype << 6)) {
#define CASE(a, b, c, d, TA, TB, TC, TD)                                                                         \
  case key3(a, b, c) | (d << 6):                                                                                 \
    return launch_fwd<true, TA, TB, TC, TD>(hidden, residual, w, new_residual, normed, rstd, rows, dim, eps, s);
    CASE(MT_BF16, MT_BF16, MT_BF16, MT_BF16, bf, bf, bf, bf)
    CASE(MT_F16, MT_F16, MT_F16, MT_F16, hf, hf, hf, hf)
    CASE(MT_F32, MT_F32, MT_F32, MT_F32, float, float, float, float)
    CASE(MT_BF16, MT_F32, MT_BF16, MT_BF16, bf, float, bf, bf)
    CASE(MT_F32, MT_F32, MT_BF16, MT_F32, float, float, bf, float)
    CASE(MT_BF16, MT_F32, MT_BF16, MT_F32, bf, float, bf, float)
#undef CASE
    default: return MT_ERR_UNSUPPORTED_DTYPE;
  }
}

static int add_rms_norm_bwd_impl(const void* new_residual, int res_dtype, const void* w, int w_dtype,
                                 const float* rstd, const void* grad_new_residual, int gres_dtype,
                                 const void* grad_normed, int gnorm_dtype, void* grad_input, int gin_dtype,
                                 void* grad_branch, void* dw, int dw_dtype, void* workspace, int64_t workspace_bytes,
                                 int64_t rows, int64_t dim, void* stream) {
  int st = validate_rows(new_residual, grad_input, rows, dim);
  if (st != MT_OK) return st;
  auto s = static_cast<cudaStream_t>(stream);
  if (rows == 0) return zero_dw(dw, dw_dtype, dim, s);
  using bf = __nv_bfloat16;
  using hf = __half;
  switch (key5(res_dtype, w_dtype, gnorm_dtype, gres_dtype, gin_dtype) | (dw_dtype << 10)) {
#define CASE(a, b, c, d, e, f, TA, TB, TC, TD, TE, TF)                                                          \
  case key5(a, b, c, d, e) | (f << 10):                                                                          \
    return launch_bwd<true, TA, TB, TC, TE, TF, TD>(new_residual, w, rstd, grad_normed, grad_new_residual,       \
                                                    grad_input, dw, workspace, workspace_bytes, rows, dim, s, 0, \
                                                    grad_branch);
    CASE(MT_BF16, MT_BF16, MT_BF16, MT_BF16, MT_BF16, MT_BF16, bf, bf, bf, bf, bf, bf)
    CASE(MT_F16, MT_F16, MT_F16, MT_F16, MT_F16, MT_F16, hf, hf, hf, hf, hf, hf)
    CASE(MT_F32, MT_F32, MT_F32, MT_F32, MT_F32, MT_F32, float, float, float, float, float, float)
    CASE(MT_BF16, MT_F32, MT_BF16, MT_BF16, MT_BF16, MT_F32, bf, float, bf, bf, bf, float)
    CASE(MT_F32, MT_F32, MT_BF16, MT_F32, MT_F32, MT_F32, float, float, bf, float, float, float)
#undef CASE
    default: return MT_ERR_UNSUPPORTED_DTYPE;
  }
}

int mt_add_rms_norm_bwd(const void* new_residual, int res_dtype, const void* w, int w_dtype, const float* rstd,
                        const void* grad_new_residual, int gres_dtype, const void* grad_normed, int gnorm_dtype,
                        void* grad_input, int gin_dtype, void* dw, int dw_dtype, void* workspace,
                        int64_t workspace_bytes, int64_t rows, int64_t dim, void* stream) {
  return add_rms_norm_bwd_impl(new_residual, res_dtype, w, w_dtype, rstd, grad_new_residual, gres_dtype, grad_normed,
                               gnorm_dtype, grad_input, gin_dtype, nullptr, dw, dw_dtype, workspace, workspace_bytes,
                               rows, dim, stream);
}

int mt_add_rms_norm_bwd_dual(const void* new_residual, int res_dtype, const void* w, int w_dtype, const float* rstd,
                             const void* grad_new_residual, int gres_dtype, const void* grad_normed, int gnorm_dtype,
                             void* grad_input, int gin_dtype, void* grad_branch, void* dw, int dw_dtype,
                             void* workspace, int64_t workspace_bytes, int64_t rows, int64_t dim, void* stream) {
  if (grad_branch == nullptr && rows > 0) return MT_ERR_INVALID_ARGUMENT;
  return add_rms_norm_bwd_impl(new_residual, res_dtype, w, w_dtype, rstd, grad_new_residual, gres_dtype, grad_normed,
                               gnorm_dtype, grad_input, gin_dtype, grad_branch, dw, dw_dtype, workspace,
                               workspace_bytes, rows, dim, stream);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// RMSNorm backward without caller-provided scratch.
//
// For callers that cannot allocate device memory at the call site, the dW
// partial sums live in this file-scope device array instead of a workspace.
// Its capacity bounds the launch: at most kNoAllocBlocks blocks of per-block
// partial rows of at most kNoAllocMaxDim floats (4 MiB, held by every GPU that
// loads the library until the process exits).  Every block overwrites its own
// partial row completely before the second stage reads it, so nothing has to
// be cleared between calls; two calls that overlap on the GPU would share the
// array and race.
// ---------------------------------------------------------------------------
namespace mt {
namespace {

constexpr int kNoAllocBlocks = 256;
constexpr int kNoAllocMaxDim = 4096;

static __device__ __align__(256) float g_rms_bwd_noalloc_partial[kNoAllocBlocks * kNoAllocMaxDim];

constexpr int kMaxNoAllocDevices = 64;
float* g_noalloc_addr[kMaxNoAllocDevices];
std::mutex g_noalloc_mutex;

// The array's name is only a host-side stand-in; the kernels need the device
// address, looked up once per device with that device current.
int noalloc_scratch(const void* any_device_ptr, float** out) {
  int st = bind_device_of(any_device_ptr);
  if (st != MT_OK) return st;
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) {
    set_last_error("cudaGetDevice", err);
    return MT_ERR_LAUNCH;
  }
  if (dev < 0 || dev >= kMaxNoAllocDevices) {
    set_last_error_text("mt_rms_norm_bwd_noalloc: device index beyond the library's per-device table (64)");
    return MT_ERR_INVALID_ARGUMENT;
  }
  // The scratch address is per device: the tensors must live on the current
  // device, or the kernel would run there with another device's array.
  cudaPointerAttributes attr;
  err = cudaPointerGetAttributes(&attr, any_device_ptr);
  if (err != cudaSuccess) {
    set_last_error("mt_rms_norm_bwd_noalloc: cudaPointerGetAttributes(x)", err);
    return MT_ERR_INVALID_ARGUMENT;
  }
  if (attr.type != cudaMemoryTypeDevice) {
    set_last_error_text("mt_rms_norm_bwd_noalloc: x is not device memory");
    return MT_ERR_INVALID_ARGUMENT;
  }
  if (attr.device != dev) {
    set_last_error_text("mt_rms_norm_bwd_noalloc: x lives on another device than the current one; "
                        "make the tensors' device current before the call");
    return MT_ERR_INVALID_ARGUMENT;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_addr[dev] == nullptr) {
    void* ptr = nullptr;
    err = cudaGetSymbolAddress(&ptr, g_rms_bwd_noalloc_partial);
    if (err != cudaSuccess || ptr == nullptr) {
      set_last_error("cudaGetSymbolAddress(rms_norm_bwd no-alloc scratch)", err);
      return MT_ERR_LAUNCH;
    }
    g_noalloc_addr[dev] = static_cast<float*>(ptr);
  }
  *out = g_noalloc_addr[dev];
  return MT_OK;
}

}  // namespace
}  // namespace mt

extern "C" int mt_rms_norm_bwd_noalloc(const void* x, int x_dtype, const void* w, int w_dtype, const float* rstd,
                                       const void* dy, int dy_dtype, void* dx, int dx_dtype, void* dw, int dw_dtype,
                                       int64_t rows, int64_t dim, void* stream) {
  int st = validate_rows(x, dx, rows, dim);
  if (st != MT_OK) return st;
  if (dim > kNoAllocMaxDim) {
    mt::set_last_error_text("mt_rms_norm_bwd_noalloc: dim exceeds the built-in scratch limit of 4096");
    return MT_ERR_WORKSPACE;
  }
  auto s = static_cast<cudaStream_t>(stream);
  if (rows == 0) return zero_dw(dw, dw_dtype, dim, s);
  float* scratch = nullptr;
  if ((st = noalloc_scratch(x, &scratch)) != MT_OK) return st;
  const int64_t cap_bytes = int64_t(kNoAllocBlocks) * kNoAllocMaxDim * 4;
  using bf = __nv_bfloat16;
  using hf = __half;
  switch (key5(x_dtype, w_dtype, dy_dtype, dx_dtype, dw_dtype)) {
#define CASE(a, b, c, d, e, TA, TB, TC, TD, TE)                                                                   \
  case key5(a, b, c, d, e):                                                                                        \
    return launch_bwd<false, TA, TB, TC, TC, TD, TE>(x, w, rstd, dy, nullptr, dx, dw, scratch, cap_bytes, rows, dim, \
                                                     s, kNoAllocBlocks);
    CASE(MT_BF16, MT_BF16, MT_BF16, MT_BF16, MT_BF16, bf, bf, bf, bf, bf)
    CASE(MT_F16, MT_F16, MT_F16, MT_F16, MT_F16, hf, hf, hf, hf, hf)
    CASE(MT_F32, MT_F32, MT_F32, MT_F32, MT_F32, float, float, float, float, float)
    CASE(MT_BF16, MT_F32, MT_BF16, MT_BF16, MT_F32, bf, float, bf, bf, float)
    CASE(MT_F16, MT_F32, MT_F16, MT_F16, MT_F32, hf, float, hf, hf, float)
    CASE(MT_F32, MT_F32, MT_BF16, MT_F32, MT_F32, float, float, bf, float, float)
#undef CASE
    default: return MT_ERR_UNSUPPORTED_DTYPE;
  }
}
