// Memory-bound transformer kernels for sm_100a: RMSNorm, RoPE, SwiGLU.
//
// All kernels move data in 16-byte vectors (8 bf16) and keep statistics in fp32.  Numerics
// follow the LLaMA reference layer (HF LlamaRMSNorm / apply_rotary_pos_emb / LlamaMLP):
//   RMSNorm  y = w * bf16(x * rsqrt(mean(x^2) + eps))
//   RoPE     rotate-half convention, cos/sin tables in bf16
//   SwiGLU   h = silu(g) * u
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
__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = (threadIdx.x < NT / 32) ? red[threadIdx.x] : 0.f;
  if (w == 0) r = warp_sum(r);
  if (threadIdx.x == 0) red[0] = r;
  __syncthreads();
  r = red[0];
  __syncthreads();
  return r;
}

// ---------------------------------------------------------------- RMSNorm
// One block per row; each thread keeps up to VPT 8-wide vectors of the row in registers.
template <int NT, int VPT>
__global__ void __launch_bounds__(NT) rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x,
                                                         const __nv_bfloat16* __restrict__ w,
                                                         __nv_bfloat16* __restrict__ y,
                                                         float* __restrict__ rstd_out, int H,
                                                         int64_t ldx, int64_t ldy, float eps) {
  __shared__ float red[NT / 32];
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * ldx;
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (threadIdx.x + i * NT) * 8;
    if (c < H) {
      load8(xr + c, v[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
    }
  }
  ss = block_sum<NT>(ss, red);
  const float rstd = rsqrtf(ss / H + eps);
  if (threadIdx.x == 0 && rstd_out) rstd_out[row] = rstd;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (threadIdx.x + i * NT) * 8;
    if (c < H) {
      float wv[8], o[8];
      load8(w + c, wv);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = wv[j] * bf16r(v[i][j] * rstd);
      store8(y + row * ldy + c, o);
    }
  }
}

// dx = rstd * (dn - n * mean(dn * n)),  dn = dy * w,  n = x * rstd
// dw += sum_rows dy * bf16(n)   (per-thread column partials, one 16-byte fp32 atomic per
// 4 columns at the end of the block)
// Each block walks a contiguous run of rows; the next row's x / dy vectors are loaded into
// registers before the current row's block reduction, so HBM latency overlaps the reduction
// and the dx stores instead of serialising with them.
template <int NT, int VPT>
__global__ void __launch_bounds__(NT) rmsnorm_bwd_kernel(
    const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
    const __nv_bfloat16* __restrict__ w, const float* __restrict__ rstd,
    __nv_bfloat16* __restrict__ dx, float* __restrict__ dw_acc, int T, int H, int64_t ldx,
    int64_t lddy, int64_t lddx, int rows_per_block, int dw_vec) {
  __shared__ float red[NT / 32];
  float dwp[VPT][8];
#pragma unroll
  for (int i = 0; i < VPT; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) dwp[i][j] = 0.f;
  float wv[VPT][8];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (threadIdx.x + i * NT) * 8;
    if (c < H) load8(w + c, wv[i]);
  }
  const int r0 = blockIdx.x * rows_per_block;
  const int r1 = min(T, r0 + rows_per_block);
  uint4 xq[VPT], gq[VPT];   // raw bf16 vectors of the row being processed
  auto fetch = [&](int row) {
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = (threadIdx.x + i * NT) * 8;
      if (c < H && row < r1) {
        xq[i] = *reinterpret_cast<const uint4*>(x + (int64_t)row * ldx + c);
        gq[i] = *reinterpret_cast<const uint4*>(dy + (int64_t)row * lddy + c);
      }
    }
  };
  auto unpack8 = [](const uint4& q, float* v) {
    float2 f;
    f = unpack_bf16x2(q.x); v[0] = f.x; v[1] = f.y;
    f = unpack_bf16x2(q.y); v[2] = f.x; v[3] = f.y;
    f = unpack_bf16x2(q.z); v[4] = f.x; v[5] = f.y;
    f = unpack_bf16x2(q.w); v[6] = f.x; v[7] = f.y;
  };
  if (r0 < r1) fetch(r0);
  for (int row = r0; row < r1; ++row) {
    const float rs = rstd[row];
    float xv[VPT][8], gv[VPT][8];
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      unpack8(xq[i], xv[i]);
      unpack8(gq[i], gv[i]);
    }
    fetch(row + 1);  // in flight during the reduction below
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = (threadIdx.x + i * NT) * 8;
      if (c < H) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float n = xv[i][j] * rs;
          const float dn = gv[i][j] * wv[i][j];
          dot += dn * n;
          dwp[i][j] += gv[i][j] * bf16r(n);
        }
      }
    }
    dot = block_sum<NT>(dot, red) / H;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = (threadIdx.x + i * NT) * 8;
      if (c < H) {
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float n = xv[i][j] * rs;
          o[j] = rs * (gv[i][j] * wv[i][j] - n * dot);
        }
        store8(dx + (int64_t)row * lddx + c, o);
      }
    }
  }
  if (r0 >= r1) return;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (threadIdx.x + i * NT) * 8;
    if (c < H) {
      if (dw_vec) {
        atomicAdd(reinterpret_cast<float4*>(dw_acc + c),
                  make_float4(dwp[i][0], dwp[i][1], dwp[i][2], dwp[i][3]));
        atomicAdd(reinterpret_cast<float4*>(dw_acc + c + 4),
                  make_float4(dwp[i][4], dwp[i][5], dwp[i][6], dwp[i][7]));
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) atomicAdd(dw_acc + c + j, dwp[i][j]);
      }
    }
  }
}

// ---------------------------------------------------------------- RoPE
// In-place rotation of the first `nheads` heads of each row of `qk` ([T, ld] with heads of
// size D laid out contiguously).  cos/sin: [max_pos, D/2] bf16; pos: [T] int32 positions.
// inverse=true applies the transpose rotation (backward).
__global__ void rope_kernel(__nv_bfloat16* __restrict__ qk, const __nv_bfloat16* __restrict__ cos_t,
                            const __nv_bfloat16* __restrict__ sin_t, const int* __restrict__ pos,
                            int T, int nheads, int D, int64_t ld, int seq_len, bool inverse) {
  const int half = D / 2;
  const int vec_per_head = half / 8;
  const int64_t total = (int64_t)T * nheads * vec_per_head;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int v = idx % vec_per_head;
    const int64_t th = idx / vec_per_head;
    const int h = th % nheads;
    const int t = th / nheads;
    const int p = pos ? pos[t] : (t % seq_len);
    __nv_bfloat16* base = qk + (int64_t)t * ld + (int64_t)h * D + v * 8;
    float a[8], b[8], c[8], s[8], oa[8], ob[8];
    load8(base, a);
    load8(base + half, b);
    load8(cos_t + (int64_t)p * half + v * 8, c);
    load8(sin_t + (int64_t)p * half + v * 8, s);
    if (!inverse) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        oa[j] = a[j] * c[j] - b[j] * s[j];
        ob[j] = b[j] * c[j] + a[j] * s[j];
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        oa[j] = a[j] * c[j] + b[j] * s[j];
        ob[j] = b[j] * c[j] - a[j] * s[j];
      }
    }
    store8(base, oa);
    store8(base + half, ob);
  }
}

// ---------------------------------------------------------------- SwiGLU
// gu: [T, ldgu] with gate at column c and up at column F + c.  h = silu(g) * u.
__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ h,
                                  int T, int F, int64_t ldgu, int64_t ldh) {
  const int vpr = F / 8;
  const int64_t total = (int64_t)T * vpr;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int t = idx / vpr, c = (idx % vpr) * 8;
    float g[8], u[8], o[8];
    load8(gu + (int64_t)t * ldgu + c, g);
    load8(gu + (int64_t)t * ldgu + F + c, u);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = g[j] / (1.f + __expf(-g[j])) * u[j];
    store8(h + (int64_t)t * ldh + c, o);
  }
}

// dg = dh * u * s * (1 + g * (1 - s)),  du = dh * g * s,  s = sigmoid(g).  Writes into dgu
// with the same [gate | up] column layout as gu (dgu may alias gu).
__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ dh, const __nv_bfloat16* gu,
                                  __nv_bfloat16* dgu, int T, int F, int64_t lddh, int64_t ldgu,
                                  int64_t lddgu) {
  const int vpr = F / 8;
  const int64_t total = (int64_t)T * vpr;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int t = idx / vpr, c = (idx % vpr) * 8;
    float d[8], g[8], u[8], og[8], ou[8];
    load8(dh + (int64_t)t * lddh + c, d);
    load8(gu + (int64_t)t * ldgu + c, g);
    load8(gu + (int64_t)t * ldgu + F + c, u);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float s = 1.f / (1.f + __expf(-g[j]));
      og[j] = d[j] * u[j] * s * (1.f + g[j] * (1.f - s));
      ou[j] = d[j] * g[j] * s;
    }
    store8(dgu + (int64_t)t * lddgu + c, og);
    store8(dgu + (int64_t)t * lddgu + F + c, ou);
  }
}

int grid_for(int64_t work, int threads) {
  int dev;
  cudaGetDevice(&dev);
  int sms;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int64_t g = (work + threads - 1) / threads;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(g, (int64_t)sms * 16)));
}

}  // namespace

// ------------------------------------------------------------------ host entry points
void rmsnorm_fwd(const torch::Tensor& x, const torch::Tensor& w, torch::Tensor& y,
                 torch::Tensor& rstd, double eps) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && y.stride(1) == 1);
  const int T = x.size(0), H = x.size(1);
  TORCH_CHECK(H % 8 == 0 && H <= 16384, "rmsnorm: H must be a multiple of 8 and <= 16384");
  TORCH_CHECK(w.numel() == H && w.is_contiguous());
  const c10::cuda::CUDAGuard g(x.device());
  auto st = at::cuda::getCurrentCUDAStream();
  auto xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto wp = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  auto yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  float* rp = rstd.defined() && rstd.numel() > 0 ? rstd.data_ptr<float>() : nullptr;
  if (T == 0) return;
  if (H <= 2048)
    rmsnorm_fwd_kernel<256, 1><<<T, 256, 0, st>>>(xp, wp, yp, rp, H, x.stride(0), y.stride(0), eps);
  else if (H <= 4096)
    rmsnorm_fwd_kernel<256, 2><<<T, 256, 0, st>>>(xp, wp, yp, rp, H, x.stride(0), y.stride(0), eps);
  else if (H <= 8192)
    rmsnorm_fwd_kernel<256, 4><<<T, 256, 0, st>>>(xp, wp, yp, rp, H, x.stride(0), y.stride(0), eps);
  else
    rmsnorm_fwd_kernel<256, 8><<<T, 256, 0, st>>>(xp, wp, yp, rp, H, x.stride(0), y.stride(0), eps);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void rmsnorm_bwd(const torch::Tensor& dy, const torch::Tensor& x, const torch::Tensor& w,
                 const torch::Tensor& rstd, torch::Tensor& dx, torch::Tensor& dw_acc) {
  TORCH_CHECK(dy.scalar_type() == at::kBFloat16 && x.scalar_type() == at::kBFloat16);
  TORCH_CHECK(dw_acc.scalar_type() == at::kFloat && dw_acc.is_contiguous());
  TORCH_CHECK(x.stride(1) == 1 && dy.stride(1) == 1 && dx.stride(1) == 1);
  const int T = x.size(0), H = x.size(1);
  TORCH_CHECK(H % 8 == 0 && H <= 16384);
  const c10::cuda::CUDAGuard g(x.device());
  auto st = at::cuda::getCurrentCUDAStream();
  if (T == 0) return;
  int dev, sms;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  auto a = reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr());
  auto b = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto c = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  auto d = reinterpret_cast<__nv_bfloat16*>(dx.data_ptr());
  const int dw_vec = (reinterpret_cast<uintptr_t>(dw_acc.data_ptr()) & 15) == 0 ? 1 : 0;
  // one 8-wide vector per thread up to H = 8192 (wider blocks instead of more registers per
  // thread, so two or more blocks stay resident per SM); about four blocks per SM in the grid
#define FT_RMS_BWD(NT, VPT)                                                                      \
  do {                                                                                         \
    const int blocks = std::min(T, sms * std::max(1, 4 * 256 / (NT)));                         \
    const int rpb = (T + blocks - 1) / blocks;                                                 \
    const int nb = (T + rpb - 1) / rpb;                                                        \
    rmsnorm_bwd_kernel<NT, VPT><<<nb, NT, 0, st>>>(a, b, c, rstd.data_ptr<float>(), d,         \
                                                   dw_acc.data_ptr<float>(), T, H, x.stride(0), \
                                                   dy.stride(0), dx.stride(0), rpb, dw_vec);    \
  } while (0)
  if (H <= 2048) FT_RMS_BWD(256, 1);
  else if (H <= 4096) FT_RMS_BWD(512, 1);
  else if (H <= 8192) FT_RMS_BWD(1024, 1);
  else FT_RMS_BWD(1024, 2);
#undef FT_RMS_BWD
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void rope_apply(torch::Tensor& qk, const torch::Tensor& cos_t, const torch::Tensor& sin_t,
                const c10::optional<torch::Tensor>& pos, int64_t nheads, int64_t head_dim,
                int64_t seq_len, bool inverse) {
  TORCH_CHECK(qk.scalar_type() == at::kBFloat16 && qk.stride(1) == 1 && qk.dim() == 2);
  TORCH_CHECK(head_dim % 16 == 0, "rope: head_dim must be a multiple of 16");
  TORCH_CHECK(cos_t.is_contiguous() && sin_t.is_contiguous());
  const int T = qk.size(0);
  if (T == 0 || nheads == 0) return;
  const c10::cuda::CUDAGuard g(qk.device());
  auto st = at::cuda::getCurrentCUDAStream();
  const int64_t work = (int64_t)T * nheads * (head_dim / 16);
  rope_kernel<<<grid_for(work, 256), 256, 0, st>>>(
      reinterpret_cast<__nv_bfloat16*>(qk.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(cos_t.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(sin_t.data_ptr()),
      pos.has_value() ? pos->data_ptr<int>() : nullptr, T, nheads, head_dim, qk.stride(0),
      seq_len, inverse);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void swiglu_fwd(const torch::Tensor& gu, torch::Tensor& h, int64_t F) {
  TORCH_CHECK(gu.stride(1) == 1 && h.stride(1) == 1 && F % 8 == 0);
  const int T = gu.size(0);
  if (T == 0) return;
  const c10::cuda::CUDAGuard g(gu.device());
  swiglu_fwd_kernel<<<grid_for((int64_t)T * F / 8, 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(h.data_ptr()), T, F, gu.stride(0), h.stride(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void swiglu_bwd(const torch::Tensor& dh, const torch::Tensor& gu, torch::Tensor& dgu, int64_t F) {
  TORCH_CHECK(dh.stride(1) == 1 && gu.stride(1) == 1 && dgu.stride(1) == 1 && F % 8 == 0);
  const int T = gu.size(0);
  if (T == 0) return;
  const c10::cuda::CUDAGuard g(gu.device());
  swiglu_bwd_kernel<<<grid_for((int64_t)T * F / 8, 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(dh.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(dgu.data_ptr()), T, F, dh.stride(0), gu.stride(0),
      dgu.stride(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace ft
