// ZeRO gradient reduce-scatter fused with the fp32 cast/scale and the sharded AdamW update.
//
// Every rank of a data-parallel group keeps the full (unsharded) gradient of a ZeRO unit in
// a symmetric buffer (CUDA-IPC shared, so peers address it over NVLink).  After the unit's
// last backward, the caller orders the ranks (every rank has finished writing its buffer;
// the caller uses a one-element NCCL all-reduce on the same stream, so there is no flag wait
// in this kernel and nothing here can spin), then this kernel, on each rank, for its own
// slice [base, base + n) of the unit:
//
//   g      = scale * sum_r buf_r[base + i]            P2P loads from every peer (fp32 or bf16)
//   g     += grad_shard[i]        (accumulate=1)       earlier reduce-scatters of the step
//   grad_shard[i] = g             (optional)           the fp32 gradient shard
//   AdamW (torch.optim.AdamW semantics) on master/m/v for the elements covered by a segment,
//   bf16 copy of the updated master -> param_shard[i]  (the shard peers gather next step)
//
// The reference does these as four separate passes: NCCL reduce-scatter (bf16, AVG), a cast
// into the fp32 master gradient, torch.optim.AdamW, and a cast back into the bf16 shard
// (femtotron/sharding/param_group_cluster.py:321-324, :334-358;
// femtotron/training/mixed_precision_manager.py:318-331).  Fused, each element's gradient
// crosses NVLink once and the fp32 gradient is never re-read.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cmath>
#include <vector>

#include "common.cuh"

namespace ft {

constexpr int RSA_MAX_SRC = 8;
constexpr int RSA_MAX_SEG = 24;

struct RSAdamArgs {
  const void* src[RSA_MAX_SRC];   // every rank's unit gradient buffer (peer addresses)
  int nsrc;
  int src_f32;
  int64_t base;                   // element offset of this rank's slice inside each buffer
  int64_t n;                      // slice length (multiple of 8)
  float scale;                    // 1 / dp for an average
  int accumulate;                 // add grad_shard's current value
  float* grad_shard;              // fp32 [n]: read when accumulate, written when store_grad
  int store_grad;
  // AdamW state (all [n], fp32 except p16); null master -> reduce only
  float* master;
  float* m;
  float* v;
  __nv_bfloat16* p16;
  float beta1, beta2, eps, bc1, bc2_sqrt;
  int nseg;                       // segments [start, end) of the slice with their lr / wd
  int64_t seg_start[RSA_MAX_SEG];
  int64_t seg_end[RSA_MAX_SEG];
  float seg_lr[RSA_MAX_SEG];
  float seg_wd[RSA_MAX_SEG];
};

__device__ __forceinline__ void rsa_load8(const void* p, int64_t i, bool f32, float (&f)[8]) {
  if (f32) {
    const float4* q = reinterpret_cast<const float4*>(static_cast<const float*>(p) + i);
    const float4 a = q[0], b = q[1];
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else {
    const uint4 q = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p) + i);
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 t = unpack_bf16x2(w[j]);
      f[2 * j] = t.x;
      f[2 * j + 1] = t.y;
    }
  }
}

__device__ __forceinline__ void ld8(const float* p, float (&f)[8]) {
  const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

__device__ __forceinline__ void st8(float* p, const float (&f)[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
}

// Segment holding element i (-1: none, e.g. alignment padding).  Segments are few and sorted.
__device__ __forceinline__ int rsa_segment(const RSAdamArgs& a, int64_t i) {
  for (int s = 0; s < a.nseg; ++s)
    if (i >= a.seg_start[s] && i < a.seg_end[s]) return s;
  return -1;
}

__global__ void __launch_bounds__(256) rs_adamw_kernel(const __grid_constant__ RSAdamArgs a) {
  // the peers' buffers were written by their own kernels before the ordering collective
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  const int64_t nvec = a.n / 8;
  const bool f32 = a.src_f32 != 0;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < nvec;
       v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i0 = v * 8;
    float g[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    // issue every source's loads before summing: keeps nsrc x 32 B in flight per thread
    float part[RSA_MAX_SRC][8];
#pragma unroll
    for (int r = 0; r < RSA_MAX_SRC; ++r)
      if (r < a.nsrc) rsa_load8(a.src[r], a.base + i0, f32, part[r]);
#pragma unroll
    for (int r = 0; r < RSA_MAX_SRC; ++r)
      if (r < a.nsrc) {
#pragma unroll
        for (int j = 0; j < 8; ++j) g[j] += part[r][j];
      }
#pragma unroll
    for (int j = 0; j < 8; ++j) g[j] *= a.scale;
    if (a.accumulate) {
      float prev[8];
      ld8(a.grad_shard + i0, prev);
#pragma unroll
      for (int j = 0; j < 8; ++j) g[j] += prev[j];
    }
    if (a.store_grad) st8(a.grad_shard + i0, g);
    if (a.master == nullptr) continue;
    // AdamW: p <- p * (1 - lr * wd); m, v moments; p <- p - lr / bc1 * m / (sqrt(v) / bc2_sqrt + eps)
    const int s0 = rsa_segment(a, i0), s7 = rsa_segment(a, i0 + 7);
    float p[8], m[8], vv[8];
    ld8(a.master + i0, p);
    ld8(a.m + i0, m);
    ld8(a.v + i0, vv);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int s = (s0 == s7) ? s0 : rsa_segment(a, i0 + j);
      if (s < 0) continue;
      const float lr = a.seg_lr[s];
      p[j] *= 1.f - lr * a.seg_wd[s];
      m[j] = a.beta1 * m[j] + (1.f - a.beta1) * g[j];
      vv[j] = a.beta2 * vv[j] + (1.f - a.beta2) * g[j] * g[j];
      p[j] -= (lr / a.bc1) * m[j] / (sqrtf(vv[j]) / a.bc2_sqrt + a.eps);
    }
    st8(a.master + i0, p);
    st8(a.m + i0, m);
    st8(a.v + i0, vv);
    uint4 o;
    o.x = pack_bf16x2(p[0], p[1]);
    o.y = pack_bf16x2(p[2], p[3]);
    o.z = pack_bf16x2(p[4], p[5]);
    o.w = pack_bf16x2(p[6], p[7]);
    *reinterpret_cast<uint4*>(a.p16 + i0) = o;
  }
}

namespace {
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
}  // namespace

// Reduce-scatter (+ optional fused AdamW) of one unit slice.  `src_ptrs` are device addresses
// of every rank's full gradient buffer (the local one included); `base` is this rank's slice
// offset (elements).  Pass an empty `master` to only reduce into grad_shard.  `segments` is a
// [nseg, 4] float64 CPU tensor of (start, end, lr, weight_decay) rows over the slice.
void rs_adamw(const std::vector<int64_t>& src_ptrs, int64_t base, int64_t n, bool src_f32,
              double scale, bool accumulate, torch::Tensor& grad_shard, bool store_grad,
              const c10::optional<torch::Tensor>& master, const c10::optional<torch::Tensor>& m,
              const c10::optional<torch::Tensor>& v, const c10::optional<torch::Tensor>& p16,
              const c10::optional<torch::Tensor>& segments, double beta1, double beta2,
              double eps, int64_t step) {
  const int nsrc = static_cast<int>(src_ptrs.size());
  TORCH_CHECK(nsrc >= 1 && nsrc <= RSA_MAX_SRC, "rs_adamw: 1..8 sources");
  TORCH_CHECK(n % 8 == 0 && n >= 0, "rs_adamw: slice length must be a multiple of 8");
  // grad_shard is read when accumulating and written when store_grad; otherwise it may be empty
  if (accumulate || store_grad)
    TORCH_CHECK(grad_shard.scalar_type() == at::kFloat && grad_shard.is_contiguous() &&
                grad_shard.numel() >= n && aligned16(grad_shard.data_ptr()),
                "rs_adamw: grad_shard must be fp32, contiguous, 16-byte aligned, >= n");
  RSAdamArgs a{};
  const int64_t es = src_f32 ? 4 : 2;
  for (int r = 0; r < nsrc; ++r) {
    a.src[r] = reinterpret_cast<const void*>(src_ptrs[r]);
    TORCH_CHECK(((src_ptrs[r] + base * es) & 15) == 0, "rs_adamw: sources must be 16-byte aligned");
  }
  a.nsrc = nsrc;
  a.src_f32 = src_f32 ? 1 : 0;
  a.base = base;
  a.n = n;
  a.scale = static_cast<float>(scale);
  a.accumulate = accumulate ? 1 : 0;
  a.grad_shard = (accumulate || store_grad) ? grad_shard.data_ptr<float>() : nullptr;
  a.store_grad = store_grad ? 1 : 0;
  if (master.has_value() && master->defined() && master->numel() > 0) {
    TORCH_CHECK(m.has_value() && v.has_value() && p16.has_value() && segments.has_value(),
                "rs_adamw: the update needs master, m, v, p16 and segments");
    for (const torch::Tensor* t : {&*master, &*m, &*v}) {
      TORCH_CHECK(t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() >= n &&
                  aligned16(t->data_ptr()), "rs_adamw: master/m/v must be fp32, contiguous, aligned");
    }
    TORCH_CHECK(p16->scalar_type() == at::kBFloat16 && p16->is_contiguous() && p16->numel() >= n &&
                aligned16(p16->data_ptr()), "rs_adamw: p16 must be bf16, contiguous, aligned");
    auto seg = segments->to(torch::kCPU, torch::kDouble).contiguous();
    TORCH_CHECK(seg.dim() == 2 && seg.size(1) == 4 && seg.size(0) <= RSA_MAX_SEG,
                "rs_adamw: segments must be [<=24, 4]");
    const double* sp = seg.data_ptr<double>();
    a.nseg = static_cast<int>(seg.size(0));
    for (int s = 0; s < a.nseg; ++s) {
      a.seg_start[s] = static_cast<int64_t>(sp[4 * s]);
      a.seg_end[s] = static_cast<int64_t>(sp[4 * s + 1]);
      a.seg_lr[s] = static_cast<float>(sp[4 * s + 2]);
      a.seg_wd[s] = static_cast<float>(sp[4 * s + 3]);
      TORCH_CHECK(a.seg_start[s] >= 0 && a.seg_end[s] <= n && a.seg_start[s] <= a.seg_end[s],
                  "rs_adamw: segment out of range");
    }
    TORCH_CHECK(step >= 1, "rs_adamw: step must be >= 1");
    a.master = master->data_ptr<float>();
    a.m = m->data_ptr<float>();
    a.v = v->data_ptr<float>();
    a.p16 = reinterpret_cast<__nv_bfloat16*>(p16->data_ptr());
    a.beta1 = static_cast<float>(beta1);
    a.beta2 = static_cast<float>(beta2);
    a.eps = static_cast<float>(eps);
    a.bc1 = static_cast<float>(1.0 - std::pow(beta1, static_cast<double>(step)));
    a.bc2_sqrt = static_cast<float>(std::sqrt(1.0 - std::pow(beta2, static_cast<double>(step))));
  }
  if (n == 0) return;
  const c10::cuda::CUDAGuard g(grad_shard.device());
  int dev, sms;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t nvec = n / 8;
  // several 256-thread blocks per SM keep enough peer loads in flight to cover NVLink latency
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((nvec + 255) / 256, 4 * sms)));
  rs_adamw_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace ft
