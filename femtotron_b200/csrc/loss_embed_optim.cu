// sm_100a kernels for the model boundaries and the optimizer:
//   * vocab-parallel cross-entropy (per-row max / sum-exp / target-logit partials, and the
//     in-place logits -> dlogits backward), so full-vocab logits are never gathered;
//   * vocab-parallel embedding lookup and its scatter-add backward;
//   * multi-tensor AdamW (fp32 master, m, v; bf16 or fp32 gradient; optional bf16 param
//     write-back) and multi-tensor sum of squares for gradient-norm clipping.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace ft {

namespace {

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float* v) {
  uint4 q = *reinterpret_cast<const uint4*>(p);
  float2 f;
  f = unpack_bf16x2(q.x); v[0] = f.x; v[1] = f.y;
  f = unpack_bf16x2(q.y); v[2] = f.x; v[3] = f.y;
  f = unpack_bf16x2(q.z); v[4] = f.x; v[5] = f.y;
  f = unpack_bf16x2(q.w); v[6] = f.x; v[7] = f.y;
}
__device__ __forceinline__ void store8(__nv_bfloat16* p, const float* v) {
  *reinterpret_cast<uint4*>(p) = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                                            pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
}

constexpr float kLog2e = 1.4426950408889634f;

// ---------------------------------------------------------------- cross-entropy
// Per row of the local vocab shard: m = max_j x_j, s = sum_j exp(x_j - m), and the target
// logit if the label falls in [vstart, vstart + V).  stats[row] = {m, s, target, has_target}.
template <int NT>
__global__ void __launch_bounds__(NT) xent_stats_kernel(const __nv_bfloat16* __restrict__ logits,
                                                        const int64_t* __restrict__ labels,
                                                        float4* __restrict__ stats, int V,
                                                        int64_t ld, int64_t vstart) {
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* x = logits + row * ld;
  float m = -INFINITY, s = 0.f;
  for (int c = threadIdx.x * 8; c < V; c += NT * 8) {
    float v[8];
    load8(x + c, v);
    float lm = v[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) lm = fmaxf(lm, v[j]);
    const float nm = fmaxf(m, lm);
    float acc = s * exp2f((m - nm) * kLog2e);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc += exp2f((v[j] - nm) * kLog2e);
    m = nm;
    s = acc;
  }
  // combine (m, s) across the warp, then across warps
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffff, m, o);
    const float os = __shfl_xor_sync(0xffffffff, s, o);
    const float nm = fmaxf(m, om);
    s = (m == -INFINITY ? 0.f : s * exp2f((m - nm) * kLog2e)) +
        (om == -INFINITY ? 0.f : os * exp2f((om - nm) * kLog2e));
    m = nm;
  }
  __shared__ float sm[NT / 32], ss[NT / 32];
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) { sm[w] = m; ss[w] = s; }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = sm[0], Ssum = ss[0];
    for (int i = 1; i < NT / 32; ++i) {
      const float nm = fmaxf(M, sm[i]);
      Ssum = (M == -INFINITY ? 0.f : Ssum * exp2f((M - nm) * kLog2e)) +
             (sm[i] == -INFINITY ? 0.f : ss[i] * exp2f((sm[i] - nm) * kLog2e));
      M = nm;
    }
    const int64_t lab = labels[row];
    float tgt = 0.f, has = 0.f;
    if (lab >= vstart && lab < vstart + V) {
      tgt = __bfloat162float(x[lab - vstart]);
      has = 1.f;
    }
    stats[row] = make_float4(M, Ssum, tgt, has);
  }
}

// dlogits = (softmax(x) - onehot(label)) * scale[row-valid] , written over the logits.
// lse[row] is the global log-sum-exp; grad_scale points at one fp32 (d loss / d row-loss).
template <int NT>
__global__ void __launch_bounds__(NT) xent_bwd_kernel(__nv_bfloat16* __restrict__ logits,
                                                      const int64_t* __restrict__ labels,
                                                      const float* __restrict__ lse,
                                                      const float* __restrict__ grad_scale, int V,
                                                      int64_t ld, int64_t vstart,
                                                      int64_t ignore_index) {
  const int64_t row = blockIdx.x;
  __nv_bfloat16* x = logits + row * ld;
  const int64_t lab = labels[row];
  const float g = (lab == ignore_index) ? 0.f : grad_scale[0];
  const float L = lse[row];
  for (int c = threadIdx.x * 8; c < V; c += NT * 8) {
    float v[8];
    load8(x + c, v);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float p = exp2f((v[j] - L) * kLog2e);
      if (vstart + c + j == lab) p -= 1.f;
      v[j] = p * g;
    }
    store8(x + c, v);
  }
}

// ---------------------------------------------------------------- embedding
__global__ void embed_fwd_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                                 __nv_bfloat16* __restrict__ out, int64_t T, int H, int64_t vstart,
                                 int64_t V) {
  const int vpr = H / 8;
  const int64_t total = T * vpr;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / vpr;
    const int c = (i % vpr) * 8;
    const int64_t id = ids[t] - vstart;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (id >= 0 && id < V) v = *reinterpret_cast<const uint4*>(table + id * H + c);
    *reinterpret_cast<uint4*>(out + t * H + c) = v;
  }
}

__global__ void embed_bwd_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ dout,
                                 float* __restrict__ dtable, int64_t T, int H, int64_t vstart,
                                 int64_t V) {
  const int vpr = H / 8;
  const int64_t total = T * vpr;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / vpr;
    const int c = (i % vpr) * 8;
    const int64_t id = ids[t] - vstart;
    if (id < 0 || id >= V) continue;
    float v[8];
    load8(dout + t * H + c, v);
    float* d = dtable + id * H + c;
#pragma unroll
    for (int j = 0; j < 8; ++j) atomicAdd(d + j, v[j]);
  }
}

// ---------------------------------------------------------------- multi-tensor AdamW
struct AdamSeg {
  float* p;             // fp32 master
  float* m;
  float* v;
  const void* g;        // gradient (bf16 or fp32)
  __nv_bfloat16* p16;   // optional bf16 copy of the updated parameter
  int64_t n;
  float wd;
  int g_f32;
  int pad;              // 1 when every array is 16-byte aligned (vector path)
};

struct AdamHyper {
  float lr, beta1, beta2, eps;
  float bc1, bc2_sqrt;   // 1 - beta1^t, sqrt(1 - beta2^t)
};

__device__ __forceinline__ void adam_elem(float& p, float& m, float& v, float g, float decay,
                                          float step_size, const AdamHyper& h) {
  p *= decay;
  m = h.beta1 * m + (1.f - h.beta1) * g;
  v = h.beta2 * v + (1.f - h.beta2) * g * g;
  p -= step_size * m / (sqrtf(v) / h.bc2_sqrt + h.eps);
}

// Blocks walk a chunk table: chunk c covers elements [start, start+len) of segment seg.
// Segments whose arrays are all 16-byte aligned (flag `pad`) move 4 elements per thread per
// iteration with 16-byte loads/stores (8-byte for bf16), which keeps enough bytes in flight
// to run near the HBM copy rate; the rest, and the ragged tail, go element by element.
__global__ void __launch_bounds__(256) adamw_kernel(const AdamSeg* __restrict__ segs,
                                                    const int2* __restrict__ chunks,
                                                    const int64_t* __restrict__ chunk_start,
                                                    AdamHyper h, const float* __restrict__ grad_scale,
                                                    int chunk_len) {
  const int2 ch = chunks[blockIdx.x];
  const AdamSeg s = segs[ch.x];
  const int64_t start = chunk_start[blockIdx.x];
  const int64_t end = min(s.n, start + chunk_len);
  const float gs = grad_scale ? grad_scale[0] : 1.f;
  const float step_size = h.lr / h.bc1;
  const float decay = 1.f - h.lr * s.wd;
  float* __restrict__ P = s.p;
  float* __restrict__ M = s.m;
  float* __restrict__ Vv = s.v;
  int64_t vec_end = start;
  if (s.pad) {
    vec_end = start + ((end - start) & ~int64_t(3));
    for (int64_t i = start + 4 * threadIdx.x; i < vec_end; i += 4 * blockDim.x) {
      float4 g4;
      if (s.g_f32) {
        g4 = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(s.g) + i);
      } else {
        const uint2 q = *reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(s.g) + i);
        const float2 a = unpack_bf16x2(q.x), b = unpack_bf16x2(q.y);
        g4 = make_float4(a.x, a.y, b.x, b.y);
      }
      float4 p4 = *reinterpret_cast<const float4*>(P + i);
      float4 m4 = *reinterpret_cast<const float4*>(M + i);
      float4 v4 = *reinterpret_cast<const float4*>(Vv + i);
      adam_elem(p4.x, m4.x, v4.x, g4.x * gs, decay, step_size, h);
      adam_elem(p4.y, m4.y, v4.y, g4.y * gs, decay, step_size, h);
      adam_elem(p4.z, m4.z, v4.z, g4.z * gs, decay, step_size, h);
      adam_elem(p4.w, m4.w, v4.w, g4.w * gs, decay, step_size, h);
      *reinterpret_cast<float4*>(P + i) = p4;
      *reinterpret_cast<float4*>(M + i) = m4;
      *reinterpret_cast<float4*>(Vv + i) = v4;
      if (s.p16)
        *reinterpret_cast<uint2*>(s.p16 + i) = make_uint2(pack_bf16x2(p4.x, p4.y), pack_bf16x2(p4.z, p4.w));
    }
  }
  for (int64_t i = vec_end + threadIdx.x; i < end; i += blockDim.x) {
    float g = s.g_f32 ? reinterpret_cast<const float*>(s.g)[i]
                      : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(s.g)[i]);
    float p = P[i], m = M[i], v = Vv[i];
    adam_elem(p, m, v, g * gs, decay, step_size, h);
    P[i] = p;
    M[i] = m;
    Vv[i] = v;
    if (s.p16) s.p16[i] = __float2bfloat16_rn(p);
  }
}

struct SqSeg {
  const void* x;
  int64_t n;
  int f32;
  int out_slot;
};

// Sum of squares per output slot (fp32 atomics into out[slot]).
__global__ void sumsq_kernel(const SqSeg* __restrict__ segs, const int2* __restrict__ chunks,
                             const int64_t* __restrict__ chunk_start, float* __restrict__ out,
                             int chunk_len) {
  const int2 ch = chunks[blockIdx.x];
  const SqSeg s = segs[ch.x];
  const int64_t start = chunk_start[blockIdx.x];
  const int64_t end = min(s.n, start + chunk_len);
  float acc = 0.f;
  for (int64_t i = start + threadIdx.x; i < end; i += blockDim.x) {
    const float g = s.f32 ? reinterpret_cast<const float*>(s.x)[i]
                          : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(s.x)[i]);
    acc += g * g;
  }
  acc = warp_sum(acc);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float r = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
    r = warp_sum(r);
    if (threadIdx.x == 0) atomicAdd(out + s.out_slot, r);
  }
}

int sm_count() {
  int dev, sms;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

}  // namespace

// ------------------------------------------------------------------ host entry points
void xent_stats(const torch::Tensor& logits, const torch::Tensor& labels, torch::Tensor& stats,
                int64_t vstart) {
  TORCH_CHECK(logits.scalar_type() == at::kBFloat16 && logits.stride(1) == 1);
  TORCH_CHECK(labels.scalar_type() == at::kLong && labels.is_contiguous());
  TORCH_CHECK(stats.scalar_type() == at::kFloat && stats.is_contiguous() && stats.size(1) == 4);
  const int T = logits.size(0), V = logits.size(1);
  TORCH_CHECK(V % 8 == 0 && logits.stride(0) % 8 == 0, "xent: vocab shard must be a multiple of 8");
  if (T == 0) return;
  const c10::cuda::CUDAGuard g(logits.device());
  xent_stats_kernel<512><<<T, 512, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), labels.data_ptr<int64_t>(),
      reinterpret_cast<float4*>(stats.data_ptr<float>()), V, logits.stride(0), vstart);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void xent_bwd(torch::Tensor& logits, const torch::Tensor& labels, const torch::Tensor& lse,
              const torch::Tensor& grad_scale, int64_t vstart, int64_t ignore_index) {
  TORCH_CHECK(logits.scalar_type() == at::kBFloat16 && logits.stride(1) == 1);
  const int T = logits.size(0), V = logits.size(1);
  TORCH_CHECK(V % 8 == 0);
  if (T == 0) return;
  const c10::cuda::CUDAGuard g(logits.device());
  xent_bwd_kernel<512><<<T, 512, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(logits.data_ptr()), labels.data_ptr<int64_t>(),
      lse.data_ptr<float>(), grad_scale.data_ptr<float>(), V, logits.stride(0), vstart,
      ignore_index);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void embed_fwd(const torch::Tensor& ids, const torch::Tensor& table, torch::Tensor& out,
               int64_t vstart) {
  TORCH_CHECK(ids.scalar_type() == at::kLong && ids.is_contiguous());
  TORCH_CHECK(table.scalar_type() == at::kBFloat16 && table.is_contiguous() && out.is_contiguous());
  const int64_t T = ids.numel();
  const int H = table.size(1);
  TORCH_CHECK(H % 8 == 0);
  if (T == 0) return;
  const c10::cuda::CUDAGuard g(ids.device());
  const int64_t work = T * H / 8;
  const int grid = static_cast<int>(std::min<int64_t>((work + 255) / 256, sm_count() * 16));
  embed_fwd_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      ids.data_ptr<int64_t>(), reinterpret_cast<const __nv_bfloat16*>(table.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), T, H, vstart, table.size(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void embed_bwd(const torch::Tensor& ids, const torch::Tensor& dout, torch::Tensor& dtable,
               int64_t vstart) {
  TORCH_CHECK(dtable.scalar_type() == at::kFloat && dtable.is_contiguous());
  TORCH_CHECK(dout.scalar_type() == at::kBFloat16 && dout.is_contiguous());
  const int64_t T = ids.numel();
  const int H = dtable.size(1);
  if (T == 0) return;
  const c10::cuda::CUDAGuard g(ids.device());
  const int64_t work = T * H / 8;
  const int grid = static_cast<int>(std::min<int64_t>((work + 255) / 256, sm_count() * 16));
  embed_bwd_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      ids.data_ptr<int64_t>(), reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()),
      dtable.data_ptr<float>(), T, H, vstart, dtable.size(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Build a chunk table for a list of segment lengths (host side), upload with the segments.
template <typename Seg>
static void launch_chunked(const std::vector<Seg>& segs, const std::vector<int64_t>& lens,
                           int chunk_len, const torch::Device& dev,
                           std::function<void(const Seg*, const int2*, const int64_t*, int)> fn) {
  std::vector<int2> chunks;
  std::vector<int64_t> starts;
  for (size_t i = 0; i < segs.size(); ++i)
    for (int64_t s = 0; s < lens[i]; s += chunk_len) {
      chunks.push_back(make_int2(static_cast<int>(i), 0));
      starts.push_back(s);
    }
  if (chunks.empty()) return;
  const size_t seg_bytes = segs.size() * sizeof(Seg);
  const size_t ch_bytes = chunks.size() * sizeof(int2);
  const size_t st_bytes = starts.size() * sizeof(int64_t);
  auto host = torch::empty({static_cast<int64_t>(seg_bytes + ch_bytes + st_bytes + 32)},
                           torch::dtype(torch::kUInt8).pinned_memory(true));
  uint8_t* hp = host.data_ptr<uint8_t>();
  size_t o_ch = (seg_bytes + 15) & ~size_t(15), o_st = (o_ch + ch_bytes + 15) & ~size_t(15);
  memcpy(hp, segs.data(), seg_bytes);
  memcpy(hp + o_ch, chunks.data(), ch_bytes);
  memcpy(hp + o_st, starts.data(), st_bytes);
  auto devbuf = host.to(dev, /*non_blocking=*/true);
  uint8_t* dp = devbuf.data_ptr<uint8_t>();
  fn(reinterpret_cast<const Seg*>(dp), reinterpret_cast<const int2*>(dp + o_ch),
     reinterpret_cast<const int64_t*>(dp + o_st), static_cast<int>(chunks.size()));
}

void adamw_multi(const std::vector<torch::Tensor>& params, const std::vector<torch::Tensor>& ms,
                 const std::vector<torch::Tensor>& vs, const std::vector<torch::Tensor>& grads,
                 const std::vector<torch::Tensor>& p16s, const std::vector<double>& wds,
                 double lr, double beta1, double beta2, double eps, int64_t step,
                 const c10::optional<torch::Tensor>& grad_scale) {
  const size_t n = params.size();
  TORCH_CHECK(ms.size() == n && vs.size() == n && grads.size() == n && wds.size() == n);
  TORCH_CHECK(p16s.empty() || p16s.size() == n);
  if (n == 0) return;
  std::vector<AdamSeg> segs(n);
  std::vector<int64_t> lens(n);
  for (size_t i = 0; i < n; ++i) {
    TORCH_CHECK(params[i].scalar_type() == at::kFloat && params[i].is_contiguous());
    TORCH_CHECK(ms[i].is_contiguous() && vs[i].is_contiguous() && grads[i].is_contiguous());
    TORCH_CHECK(grads[i].numel() == params[i].numel());
    segs[i].p = params[i].data_ptr<float>();
    segs[i].m = ms[i].data_ptr<float>();
    segs[i].v = vs[i].data_ptr<float>();
    segs[i].g = grads[i].data_ptr();
    segs[i].g_f32 = grads[i].scalar_type() == at::kFloat ? 1 : 0;
    segs[i].p16 = (!p16s.empty() && p16s[i].defined() && p16s[i].numel() == params[i].numel())
                      ? reinterpret_cast<__nv_bfloat16*>(p16s[i].data_ptr())
                      : nullptr;
    segs[i].n = params[i].numel();
    segs[i].wd = static_cast<float>(wds[i]);
    auto al = [](const void* q, uintptr_t a) { return (reinterpret_cast<uintptr_t>(q) & (a - 1)) == 0; };
    segs[i].pad = (al(segs[i].p, 16) && al(segs[i].m, 16) && al(segs[i].v, 16) &&
                   al(segs[i].g, segs[i].g_f32 ? 16 : 8) && (!segs[i].p16 || al(segs[i].p16, 8)))
                      ? 1 : 0;
    lens[i] = segs[i].n;
  }
  const c10::cuda::CUDAGuard g(params[0].device());
  auto st = at::cuda::getCurrentCUDAStream();
  AdamHyper h;
  h.lr = lr; h.beta1 = beta1; h.beta2 = beta2; h.eps = eps;
  h.bc1 = 1.0 - std::pow(beta1, static_cast<double>(step));
  h.bc2_sqrt = std::sqrt(1.0 - std::pow(beta2, static_cast<double>(step)));
  const float* gsp = grad_scale.has_value() ? grad_scale->data_ptr<float>() : nullptr;
  constexpr int CH = 1 << 16;
  launch_chunked<AdamSeg>(segs, lens, CH, params[0].device(),
                          [&](const AdamSeg* s, const int2* c, const int64_t* o, int nc) {
                            adamw_kernel<<<nc, 256, 0, st>>>(s, c, o, h, gsp, CH);
                          });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// out[slot] += sum(x_i^2) for every tensor i assigned to `slot`.
void sumsq_multi(const std::vector<torch::Tensor>& xs, const std::vector<int64_t>& slots,
                 torch::Tensor& out) {
  const size_t n = xs.size();
  if (n == 0) return;
  TORCH_CHECK(slots.size() == n && out.scalar_type() == at::kFloat);
  std::vector<SqSeg> segs(n);
  std::vector<int64_t> lens(n);
  for (size_t i = 0; i < n; ++i) {
    TORCH_CHECK(xs[i].is_contiguous());
    segs[i].x = xs[i].data_ptr();
    segs[i].n = xs[i].numel();
    segs[i].f32 = xs[i].scalar_type() == at::kFloat ? 1 : 0;
    segs[i].out_slot = static_cast<int>(slots[i]);
    lens[i] = segs[i].n;
  }
  const c10::cuda::CUDAGuard g(xs[0].device());
  auto st = at::cuda::getCurrentCUDAStream();
  constexpr int CH = 1 << 16;
  float* op = out.data_ptr<float>();
  launch_chunked<SqSeg>(segs, lens, CH, xs[0].device(),
                        [&](const SqSeg* s, const int2* c, const int64_t* o, int nc) {
                          sumsq_kernel<<<nc, 512, 0, st>>>(s, c, o, op, CH);
                        });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace ft
