// Fused AdamW on fp32 master weights that also writes each parameter's 16-bit
// copy (the operand the GEMMs read), in one pass over the optimizer state.
//
// Reference semantics (duoan/mega-trading): the optimizer is
// torch.optim.AdamW(fused=True) (src/mega_trading/trainer.py:535-545):
// decoupled weight decay (Loshchilov & Hutter), bias-corrected moments,
//   p <- p - lr * wd * p
//   m <- b1 m + (1 - b1) g ;  v <- b2 v + (1 - b2) g^2
//   p <- p - (lr / (1 - b1^t)) * m / (sqrt(v) / sqrt(1 - b2^t) + eps)
// The reference then casts the fp32 weights to bf16 inside every autocast
// forward; here the cast happens once per step, in this kernel, straight into
// the packed layouts the projection GEMMs read (q/k/v rows stacked, gate/up
// rows interleaved in blocks).
//
// B200 design: all parameters in one launch.  The host passes a device table
// of tensors with prefix offsets; each block takes 2048 consecutive elements
// of the flattened parameter space, finds its first tensor by binary search
// and walks forward, 8 independent elements per thread (coalesced fp32
// streams: 28 B read/written per element plus the 2 B copy -- HBM-bound).
#include "common.cuh"

namespace mt {
namespace {

constexpr int kOptThreads = 256;
constexpr int kOptPerThread = 8;
constexpr int kOptChunk = kOptThreads * kOptPerThread;

struct AdamWArgs {
  float lr_wd;       // lr * weight_decay
  float beta1, beta2;
  float eps;
  float step_size;   // lr / (1 - beta1^t)
  float bc2_sqrt;    // sqrt(1 - beta2^t)
  const uint32_t* guard;  // device status word: nonzero -> leave everything untouched
};

__device__ __forceinline__ int find_tensor(const MtAdamWTensor* __restrict__ t, int n, int64_t i) {
  int lo = 0, hi = n - 1;  // last tensor with offset <= i
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (t[mid].offset <= i)
      lo = mid;
    else
      hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ void adamw_update(float& p, float g, float& m, float& v, const AdamWArgs& a) {
  p -= a.lr_wd * p;
  m = fmaf(a.beta1, m, (1.f - a.beta1) * g);
  v = fmaf(a.beta2, v, (1.f - a.beta2) * g * g);
  const float denom = sqrtf(v) / a.bc2_sqrt + a.eps;
  p -= a.step_size * (m / denom);
}

template <typename TS>
__device__ __forceinline__ void store_shadow(const MtAdamWTensor& d, int64_t j, float p) {
  if (d.shadow == nullptr) return;
  int64_t s = j;
  if (d.shadow_block != d.numel) {
    const uint32_t blk = (uint32_t)d.shadow_block;  // < 2^32 (checked on the host)
    const uint32_t q = (uint32_t)j / blk;
    s = int64_t(q) * d.shadow_stride + ((uint32_t)j - q * blk);
  }
  static_cast<TS*>(d.shadow)[s] = from_f32<TS>(p);
}

template <typename TS>
__global__ void __launch_bounds__(kOptThreads) adamw_kernel(const MtAdamWTensor* __restrict__ tab, int n_tensors,
                                                            int64_t total, AdamWArgs a) {
  const int64_t base = int64_t(blockIdx.x) * kOptChunk;
  if (base >= total) return;
  // a kernel of this step reported a device error: its gradients may be
  // partial, so no weight, moment or copy is changed
  if (a.guard != nullptr && *a.guard != 0u) return;
  int t = find_tensor(tab, n_tensors, base);
  const MtAdamWTensor d = tab[t];
  if (base + kOptChunk <= d.offset + d.numel) {
    // the whole chunk lies in one tensor: all loads first, then the updates
    const int64_t j0 = base - d.offset + threadIdx.x;
    float p[kOptPerThread], g[kOptPerThread], m[kOptPerThread], v[kOptPerThread];
#pragma unroll
    for (int k = 0; k < kOptPerThread; ++k) {
      const int64_t j = j0 + k * kOptThreads;
      p[k] = d.param[j];
      g[k] = d.grad[j];
      m[k] = d.exp_avg[j];
      v[k] = d.exp_avg_sq[j];
    }
#pragma unroll
    for (int k = 0; k < kOptPerThread; ++k) {
      const int64_t j = j0 + k * kOptThreads;
      adamw_update(p[k], g[k], m[k], v[k], a);
      d.param[j] = p[k];
      d.exp_avg[j] = m[k];
      d.exp_avg_sq[j] = v[k];
      store_shadow<TS>(d, j, p[k]);
    }
    return;
  }
  // chunk crosses tensor boundaries (or is the last one): element by element
  for (int k = 0; k < kOptPerThread; ++k) {
    const int64_t i = base + threadIdx.x + int64_t(k) * kOptThreads;
    if (i >= total) break;
    while (t + 1 < n_tensors && tab[t + 1].offset <= i) ++t;
    const MtAdamWTensor& e = tab[t];
    const int64_t j = i - e.offset;
    float p = e.param[j], m = e.exp_avg[j], v = e.exp_avg_sq[j];
    adamw_update(p, e.grad[j], m, v, a);
    e.param[j] = p;
    e.exp_avg[j] = m;
    e.exp_avg_sq[j] = v;
    store_shadow<TS>(e, j, p);
  }
}

}  // namespace
}  // namespace mt

using namespace mt;

extern "C" int mt_adamw_step(const MtAdamWTensor* tensors, int n_tensors, int64_t total, int shadow_dtype,
                             float lr, float beta1, float beta2, float eps, float weight_decay, float step_size,
                             float bias_correction2_sqrt, const uint32_t* skip_if_set, void* stream) {
  if (n_tensors < 0 || total < 0) return MT_ERR_INVALID_ARGUMENT;
  if (n_tensors == 0 || total == 0) return MT_OK;
  if (tensors == nullptr) return MT_ERR_INVALID_ARGUMENT;
  if (shadow_dtype != MT_BF16 && shadow_dtype != MT_F16) return MT_ERR_UNSUPPORTED_DTYPE;
  if (!(bias_correction2_sqrt > 0.f) || !(eps >= 0.f)) return MT_ERR_INVALID_ARGUMENT;
  int st = bind_device_of(tensors);
  if (st != MT_OK) return st;
  AdamWArgs a;
  a.lr_wd = lr * weight_decay;
  a.beta1 = beta1;
  a.beta2 = beta2;
  a.eps = eps;
  a.step_size = step_size;
  a.bc2_sqrt = bias_correction2_sqrt;
  a.guard = skip_if_set;
  const int64_t blocks = (total + kOptChunk - 1) / kOptChunk;
  if (blocks > 0x7fffffff) return MT_ERR_INVALID_ARGUMENT;
  auto s = static_cast<cudaStream_t>(stream);
  if (shadow_dtype == MT_BF16)
    adamw_kernel<__nv_bfloat16><<<(unsigned)blocks, kOptThreads, 0, s>>>(tensors, n_tensors, total, a);
  else
    adamw_kernel<__half><<<(unsigned)blocks, kOptThreads, 0, s>>>(tensors, n_tensors, total, a);
  return check_launch("adamw_step");
}
