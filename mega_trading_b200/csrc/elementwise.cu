// RoPE (interleaved pairs) and the SwiGLU gate, forward and backward.
//
// Reference semantics (duoan/mega-trading):
//   RoPE   src/mega_trading/kernels/triton_ops.py:45-54, :187-214, :477-525,
//          :690-761; torch path model.py:312-316 (_rotate).  Tables arrive
//          already rounded to the activation dtype (model.py:290-291).
//   SwiGLU triton_ops.py:57-61, :431-474, :774-782, :799-819; torch path
//          F.silu(g) * u (model.py:255).
//
// B200 design: pure HBM streaming.  Each thread moves 16 bytes per tensor per
// step (8 bf16/fp16 elements = 4 RoPE pairs), math in fp32 with one rounding
// per output, grid-stride loops sized to a multiple of the SM count.
#include <algorithm>

#include "common.cuh"

namespace mt {
namespace {

constexpr int kThreads = 256;

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Blocks for `units` one-per-thread work items, at most `max_waves` full waves
// (8 blocks of 256 threads per SM) with grid-stride loops beyond that.
// Measured side by side on the config-2 shapes (65,536 x 2048): the packed
// SwiGLU kernels and the plain backward run 6-7 % faster with one item per
// thread than with a 4-wave grid, the plain forward 12 % slower (it keeps 4
// waves); RoPE is within 1 % either way (8 waves).
int grid_for(int64_t units, int64_t max_waves) {
  const int64_t per_wave = int64_t(get_sm_count()) * 8;
  int64_t blocks = (units + kThreads - 1) / kThreads;
  blocks = std::min<int64_t>(blocks, std::min<int64_t>(per_wave * max_waves, int64_t(1) << 30));
  return (int)(blocks < 1 ? 1 : blocks);
}
constexpr int64_t kRopeWaves = 8;
constexpr int64_t kSwigluWaves = int64_t(1) << 20;
constexpr int64_t kSwigluFwdWaves = 4;

template <typename F>
int with_half_dtype(int code, F&& f) {
  switch (code) {
    case MT_F32: return f(float{});
    case MT_F16: return f(__half{});
    case MT_BF16: return f(__nv_bfloat16{});
    default: return MT_ERR_UNSUPPORTED_DTYPE;
  }
}

// ---------------------------------------------------------------------------
// RoPE
// ---------------------------------------------------------------------------
struct RopeArgs {
  const void* in[2];
  void* out[2];
  int64_t heads[2];
  int64_t is[2][4];  // input strides (b, h, t, d) in elements
  int64_t os[2][4];  // output strides
  const void* cos;
  const void* sin;
  int64_t cs[2];  // table strides (t, i)
  int64_t ss[2];
  int64_t B, T, half;
  float sign;  // -1 for the backward (rotation by -theta)
};

// Vector path: stride_d == 1 for inputs and outputs, D % 8 == 0, table inner
// stride 1.  Unit = 4 pairs (8 elements) of one (b, h, t) row; unit indices
// fit in 32 bits and are decomposed with precomputed divisors.  HEAD_INNER
// walks the heads of one position before the next position: the order of
// memory when q/k are views of a projection's [B, T, heads, D] rows, so
// consecutive warps stream consecutive bytes (measured 3 % faster there than
// walking positions first).
struct RopeDivs {
  FastDiv cpr, T, heads[2];
};

template <typename T, bool HEAD_INNER>
__global__ void __launch_bounds__(kThreads) rope_vec(RopeArgs a, RopeDivs dv, uint32_t units_q, uint32_t units_total) {
  for (uint32_t u = blockIdx.x * blockDim.x + threadIdx.x; u < units_total; u += gridDim.x * blockDim.x) {
    const int which = u < units_q ? 0 : 1;
    uint32_t v = which ? u - units_q : u;
    uint32_t q = dv.cpr.div(v);
    const uint32_t c = v - q * dv.cpr.d;
    v = q;
    uint32_t t, b, h;
    if constexpr (HEAD_INNER) {
      q = dv.heads[which].div(v);
      h = v - q * dv.heads[which].d;
      v = q;
      b = dv.T.div(v);
      t = v - b * dv.T.d;
    } else {
      q = dv.T.div(v);
      t = v - q * dv.T.d;
      v = q;
      b = dv.heads[which].div(v);
      h = v - b * dv.heads[which].d;
    }
    const T* src = static_cast<const T*>(a.in[which]) + b * a.is[which][0] + h * a.is[which][1] +
                   int64_t(t) * a.is[which][2] + c * 8;
    T* dst = static_cast<T*>(a.out[which]) + b * a.os[which][0] + h * a.os[which][1] + int64_t(t) * a.os[which][2] +
             c * 8;
    const T* cp = static_cast<const T*>(a.cos) + int64_t(t) * a.cs[0] + c * 4;
    const T* sp = static_cast<const T*>(a.sin) + int64_t(t) * a.ss[0] + c * 4;
    float x[8], o[8];
    load_vec<T, 8>(src, x);
    uint2 craw = *reinterpret_cast<const uint2*>(cp);
    uint2 sraw = *reinterpret_cast<const uint2*>(sp);
    const T* ce = reinterpret_cast<const T*>(&craw);
    const T* se = reinterpret_cast<const T*>(&sraw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float cs = to_f32<T>(ce[i]);
      const float sn = a.sign * to_f32<T>(se[i]);
      const float e = x[2 * i], od = x[2 * i + 1];
      o[2 * i] = e * cs - od * sn;
      o[2 * i + 1] = e * sn + od * cs;
    }
    store_vec<T, 8>(dst, o);
  }
}

// Generic path: one pair per thread, arbitrary strides.
template <typename T>
__global__ void __launch_bounds__(kThreads) rope_scalar(RopeArgs a, int64_t units_q, int64_t units_total) {
  for (int64_t u = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; u < units_total;
       u += int64_t(gridDim.x) * blockDim.x) {
    const int which = u < units_q ? 0 : 1;
    int64_t v = which ? u - units_q : u;
    const int64_t i = v % a.half;
    v /= a.half;
    const int64_t t = v % a.T;
    v /= a.T;
    const int64_t h = v % a.heads[which];
    const int64_t b = v / a.heads[which];
    const T* src = static_cast<const T*>(a.in[which]) + b * a.is[which][0] + h * a.is[which][1] + t * a.is[which][2];
    T* dst = static_cast<T*>(a.out[which]) + b * a.os[which][0] + h * a.os[which][1] + t * a.os[which][2];
    const float cs = to_f32<T>(static_cast<const T*>(a.cos)[t * a.cs[0] + i * a.cs[1]]);
    const float sn = a.sign * to_f32<T>(static_cast<const T*>(a.sin)[t * a.ss[0] + i * a.ss[1]]);
    const float e = to_f32<T>(src[(2 * i) * a.is[which][3]]);
    const float od = to_f32<T>(src[(2 * i + 1) * a.is[which][3]]);
    dst[(2 * i) * a.os[which][3]] = from_f32<T>(e * cs - od * sn);
    dst[(2 * i + 1) * a.os[which][3]] = from_f32<T>(e * sn + od * cs);
  }
}

// ---------------------------------------------------------------------------
// SwiGLU gate
//   y  = round_T(silu(g)) * u
//   dg = dy * u * sigma(g) * (1 + g * (1 - sigma(g)))
//   du = dy * round_T(silu(g))
// ---------------------------------------------------------------------------

template <typename T>
__global__ void __launch_bounds__(kThreads) swiglu_fwd_k(const T* __restrict__ g, const T* __restrict__ u,
                                                          T* __restrict__ y, int64_t n) {
  constexpr int V = 16 / sizeof(T);
  const int64_t nvec = n / V;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < nvec; i += int64_t(gridDim.x) * blockDim.x) {
    float gv[V], uv[V], o[V];
    load_vec<T, V>(g + i * V, gv);
    load_vec<T, V>(u + i * V, uv);
#pragma unroll
    for (int j = 0; j < V; ++j) o[j] = round_to<T>(gv[j] * sigmoid_f32(gv[j])) * uv[j];
    store_vec<T, V>(y + i * V, o);
  }
  // tail (n % V elements), handled by the first threads of block 0
  if (blockIdx.x == 0) {
    const int64_t i = nvec * V + threadIdx.x;
    if (i < n) {
      const float gv = to_f32<T>(g[i]);
      y[i] = from_f32<T>(round_to<T>(gv * sigmoid_f32(gv)) * to_f32<T>(u[i]));
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) swiglu_bwd_k(const T* __restrict__ g, const T* __restrict__ u,
                                                          const T* __restrict__ dy, T* __restrict__ dg,
                                                          T* __restrict__ du, int64_t n) {
  constexpr int V = 16 / sizeof(T);
  const int64_t nvec = n / V;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < nvec; i += int64_t(gridDim.x) * blockDim.x) {
    float gv[V], uv[V], dv[V], og[V], ou[V];
    load_vec<T, V>(g + i * V, gv);
    load_vec<T, V>(u + i * V, uv);
    load_vec<T, V>(dy + i * V, dv);
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const float s = sigmoid_f32(gv[j]);
      og[j] = dv[j] * uv[j] * s * (1.f + gv[j] * (1.f - s));
      ou[j] = dv[j] * round_to<T>(gv[j] * s);
    }
    store_vec<T, V>(dg + i * V, og);
    store_vec<T, V>(du + i * V, ou);
  }
  if (blockIdx.x == 0) {
    const int64_t i = nvec * V + threadIdx.x;
    if (i < n) {
      const float gv = to_f32<T>(g[i]), uv = to_f32<T>(u[i]), dv = to_f32<T>(dy[i]);
      const float s = sigmoid_f32(gv);
      dg[i] = from_f32<T>(dv * uv * s * (1.f + gv * (1.f - s)));
      du[i] = from_f32<T>(dv * round_to<T>(gv * s));
    }
  }
}


// Packed SwiGLU: gu = [gate | up] rows of width 2 * inter (one GEMM with the
// concatenated w1 / w3 weights), y = silu(gate) * up of width inter; the
// backward writes the packed gradient [dgate | dup] for one backward GEMM.
template <typename T>
__global__ void __launch_bounds__(kThreads) swiglu_packed_fwd_k(const T* __restrict__ gu, T* __restrict__ y,
                                                                 uint32_t total, FastDiv vpr, int inter) {
  constexpr int V = 16 / sizeof(T);
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int64_t r = vpr.div(i);
    const int c = int(i - uint32_t(r) * vpr.d) * V;
    float gv[V], uv[V], o[V];
    load_vec<T, V>(gu + r * 2 * inter + c, gv);
    load_vec<T, V>(gu + r * 2 * inter + inter + c, uv);
#pragma unroll
    for (int j = 0; j < V; ++j) o[j] = round_to<T>(gv[j] * sigmoid_f32(gv[j])) * uv[j];
    store_vec<T, V>(y + r * inter + c, o);
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) swiglu_packed_bwd_k(const T* __restrict__ gu, const T* __restrict__ dy,
                                                                 T* __restrict__ dgu, uint32_t total, FastDiv vpr,
                                                                 int inter) {
  constexpr int V = 16 / sizeof(T);
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int64_t r = vpr.div(i);
    const int c = int(i - uint32_t(r) * vpr.d) * V;
    float gv[V], uv[V], dv[V], og[V], ou[V];
    load_vec<T, V>(gu + r * 2 * inter + c, gv);
    load_vec<T, V>(gu + r * 2 * inter + inter + c, uv);
    load_vec<T, V>(dy + r * inter + c, dv);
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const float s = sigmoid_f32(gv[j]);
      og[j] = dv[j] * uv[j] * s * (1.f + gv[j] * (1.f - s));
      ou[j] = dv[j] * round_to<T>(gv[j] * s);
    }
    store_vec<T, V>(dgu + r * 2 * inter + c, og);
    store_vec<T, V>(dgu + r * 2 * inter + inter + c, ou);
  }
}

}  // namespace
}  // namespace mt

using namespace mt;

extern "C" {

int mt_rope(const void* q, const void* k, const void* cos, const void* sin, void* q_out, void* k_out, int dtype,
            int64_t B, int64_t Hq, int64_t Hk, int64_t T, int64_t D, const int64_t* qs, const int64_t* ks,
            const int64_t* qos, const int64_t* kos, const int64_t* cs, const int64_t* ss, int negate_sin,
            void* stream) {
  if (B < 0 || Hq < 0 || Hk < 0 || T < 0 || D <= 0 || (D % 2) != 0) return MT_ERR_INVALID_ARGUMENT;
  if (!qs || !ks || !qos || !kos || !cs || !ss) return MT_ERR_INVALID_ARGUMENT;
  RopeArgs a;
  a.in[0] = q;
  a.in[1] = k;
  a.out[0] = q_out;
  a.out[1] = k_out;
  a.heads[0] = Hq;
  a.heads[1] = Hk;
  for (int i = 0; i < 4; ++i) {
    a.is[0][i] = qs[i];
    a.is[1][i] = ks[i];
    a.os[0][i] = qos[i];
    a.os[1][i] = kos[i];
  }
  a.cos = cos;
  a.sin = sin;
  a.cs[0] = cs[0];
  a.cs[1] = cs[1];
  a.ss[0] = ss[0];
  a.ss[1] = ss[1];
  a.B = B;
  a.T = T;
  a.half = D / 2;
  a.sign = negate_sin ? -1.f : 1.f;
  const int64_t rows_q = B * Hq * T, rows_k = B * Hk * T;
  if (rows_q + rows_k == 0) return MT_OK;
  auto s = static_cast<cudaStream_t>(stream);
  return with_half_dtype(dtype, [&](auto tv) {
    using TT = decltype(tv);
    const int vecw = 16 / (int)sizeof(TT);
    bool vec = (vecw == 8) && (D % 8 == 0) && qs[3] == 1 && ks[3] == 1 && qos[3] == 1 && kos[3] == 1 &&
               cs[1] == 1 && ss[1] == 1;
    // every row start and table row start must stay 16-byte / 8-byte aligned
    for (int i = 0; vec && i < 3; ++i)
      vec = (qs[i] % 8 == 0) && (ks[i] % 8 == 0) && (qos[i] % 8 == 0) && (kos[i] % 8 == 0);
    vec = vec && (cs[0] % 4 == 0) && (ss[0] % 4 == 0);
    vec = vec && aligned16(q) && aligned16(k) && aligned16(q_out) && aligned16(k_out) &&
          (reinterpret_cast<uintptr_t>(cos) % 8 == 0) && (reinterpret_cast<uintptr_t>(sin) % 8 == 0);
    const int64_t cpr = D / 8;
    vec = vec && (rows_q + rows_k) * cpr < (int64_t(1) << 31) && B * Hq < (int64_t(1) << 31);
    if constexpr (sizeof(TT) != 2) vec = false;
    if (vec) {
      const int64_t uq = rows_q * cpr, ut = uq + rows_k * cpr;
      RopeDivs dv;
      dv.cpr.init((uint32_t)cpr);
      dv.T.init((uint32_t)(T > 0 ? T : 1));
      dv.heads[0].init((uint32_t)(Hq > 0 ? Hq : 1));
      dv.heads[1].init((uint32_t)(Hk > 0 ? Hk : 1));
      const bool head_inner = qs[1] < qs[2] && ks[1] < ks[2] && qos[1] < qos[2] && kos[1] < kos[2];
      if constexpr (sizeof(TT) == 2) {
        if (head_inner)
          rope_vec<TT, true><<<grid_for(ut, kRopeWaves), kThreads, 0, s>>>(a, dv, (uint32_t)uq, (uint32_t)ut);
        else
          rope_vec<TT, false><<<grid_for(ut, kRopeWaves), kThreads, 0, s>>>(a, dv, (uint32_t)uq, (uint32_t)ut);
      }
    } else {
      const int64_t uq = rows_q * (D / 2), ut = uq + rows_k * (D / 2);
      rope_scalar<TT><<<grid_for(ut, kRopeWaves), kThreads, 0, s>>>(a, uq, ut);
    }
    return check_launch("rope");
  });
}

int mt_swiglu_fwd(const void* g, const void* u, void* y, int dtype, int64_t n, void* stream) {
  if (n < 0) return MT_ERR_INVALID_ARGUMENT;
  if (n == 0) return MT_OK;
  if (!aligned16(g) || !aligned16(u) || !aligned16(y)) return MT_ERR_UNSUPPORTED_LAYOUT;
  auto s = static_cast<cudaStream_t>(stream);
  return with_half_dtype(dtype, [&](auto tv) {
    using TT = decltype(tv);
    const int64_t vecs = n / (16 / (int64_t)sizeof(TT)) + 1;
    swiglu_fwd_k<TT><<<grid_for(vecs, kSwigluFwdWaves), kThreads, 0, s>>>(static_cast<const TT*>(g), static_cast<const TT*>(u),
                                                          static_cast<TT*>(y), n);
    return check_launch("swiglu_fwd");
  });
}

int mt_swiglu_bwd(const void* g, const void* u, const void* dy, void* dg, void* du, int dtype, int64_t n,
                  void* stream) {
  if (n < 0) return MT_ERR_INVALID_ARGUMENT;
  if (n == 0) return MT_OK;
  if (!aligned16(g) || !aligned16(u) || !aligned16(dy) || !aligned16(dg) || !aligned16(du))
    return MT_ERR_UNSUPPORTED_LAYOUT;
  auto s = static_cast<cudaStream_t>(stream);
  return with_half_dtype(dtype, [&](auto tv) {
    using TT = decltype(tv);
    const int64_t vecs = n / (16 / (int64_t)sizeof(TT)) + 1;
    swiglu_bwd_k<TT><<<grid_for(vecs, kSwigluWaves), kThreads, 0, s>>>(static_cast<const TT*>(g), static_cast<const TT*>(u),
                                                          static_cast<const TT*>(dy), static_cast<TT*>(dg),
                                                          static_cast<TT*>(du), n);
    return check_launch("swiglu_bwd");
  });
}


int mt_swiglu_packed_fwd(const void* gu, void* y, int dtype, int64_t rows, int64_t inter, void* stream) {
  if (rows < 0 || inter <= 0) return MT_ERR_INVALID_ARGUMENT;
  if (rows == 0) return MT_OK;
  if (dtype != MT_BF16 && dtype != MT_F16) return MT_ERR_UNSUPPORTED_DTYPE;
  if (inter % 8 != 0 || !aligned16(gu) || !aligned16(y)) return MT_ERR_UNSUPPORTED_LAYOUT;
  if (rows * inter / 8 >= (int64_t(1) << 31)) return MT_ERR_INVALID_ARGUMENT;
  auto s = static_cast<cudaStream_t>(stream);
  return with_half_dtype(dtype, [&](auto tv) {
    using TT = decltype(tv);
    if constexpr (sizeof(TT) == 2) {
      FastDiv vpr;
      vpr.init((uint32_t)(inter / 8));
      swiglu_packed_fwd_k<TT><<<grid_for(rows * inter / 8, kSwigluWaves), kThreads, 0, s>>>(
          static_cast<const TT*>(gu), static_cast<TT*>(y), (uint32_t)(rows * inter / 8), vpr, (int)inter);
    }
    return check_launch("swiglu_packed_fwd");
  });
}

int mt_swiglu_packed_bwd(const void* gu, const void* dy, void* dgu, int dtype, int64_t rows, int64_t inter,
                         void* stream) {
  if (rows < 0 || inter <= 0) return MT_ERR_INVALID_ARGUMENT;
  if (rows == 0) return MT_OK;
  if (dtype != MT_BF16 && dtype != MT_F16) return MT_ERR_UNSUPPORTED_DTYPE;
  if (inter % 8 != 0 || !aligned16(gu) || !aligned16(dy) || !aligned16(dgu)) return MT_ERR_UNSUPPORTED_LAYOUT;
  if (rows * inter / 8 >= (int64_t(1) << 31)) return MT_ERR_INVALID_ARGUMENT;
  auto s = static_cast<cudaStream_t>(stream);
  return with_half_dtype(dtype, [&](auto tv) {
    using TT = decltype(tv);
    if constexpr (sizeof(TT) == 2) {
      FastDiv vpr;
      vpr.init((uint32_t)(inter / 8));
      swiglu_packed_bwd_k<TT><<<grid_for(rows * inter / 8, kSwigluWaves), kThreads, 0, s>>>(
          static_cast<const TT*>(gu), static_cast<const TT*>(dy), static_cast<TT*>(dgu), (uint32_t)(rows * inter / 8),
          vpr, (int)inter);
    }
    return check_launch("swiglu_packed_bwd");
  });
}

}  // extern "C"
