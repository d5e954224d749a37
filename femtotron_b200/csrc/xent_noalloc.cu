// Allocation-free mean cross-entropy loss (see xent_noalloc.h for the contract).  This file
// has no counterpart in the reference framework.
//
// Two kernels run on the caller's stream: a per-row pass writes (max, sum-exp, target logit,
// valid) of every row into the file-scope scratch array, and a one-block pass reduces those
// rows into the mean loss.  The scratch array is a `static __device__` variable, so the
// library owns that memory for the life of the process and no call allocates.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <mutex>

#include "xent_noalloc.h"

namespace {

// Per-row statistics of the last call: 16 bytes per row, 1 MiB in total, on every GPU.
static __device__ __align__(256) float4 g_xent_noalloc_rows[FT_XENT_NOALLOC_MAX_ROWS];

constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ void combine(float& m, float& s, float om, float os) {
  const float nm = fmaxf(m, om);
  s = (m == -INFINITY ? 0.f : s * exp2f((m - nm) * kLog2e)) +
      (om == -INFINITY ? 0.f : os * exp2f((om - nm) * kLog2e));
  m = nm;
}

// One block per row: online max / sum-exp over the row in 8-wide bf16 vectors.
__global__ void __launch_bounds__(512) noalloc_rows_kernel(const __nv_bfloat16* __restrict__ logits,
                                                           const int64_t* __restrict__ labels,
                                                           float4* __restrict__ rows_out, int vocab,
                                                           int64_t ld, int64_t ignore_index) {
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* x = logits + row * ld;
  float m = -INFINITY, s = 0.f;
  for (int c = threadIdx.x * 8; c < vocab; c += blockDim.x * 8) {
    const uint4 q = *reinterpret_cast<const uint4*>(x + c);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&q);
    float v[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
    }
    float lm = v[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) lm = fmaxf(lm, v[j]);
    const float nm = fmaxf(m, lm);
    float acc = (m == -INFINITY) ? 0.f : s * exp2f((m - nm) * kLog2e);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc += exp2f((v[j] - nm) * kLog2e);
    m = nm;
    s = acc;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    combine(m, s, __shfl_xor_sync(0xffffffff, m, o), __shfl_xor_sync(0xffffffff, s, o));
  __shared__ float sm[16], ss[16];
  const int w = threadIdx.x / 32;
  if ((threadIdx.x & 31) == 0) {
    sm[w] = m;
    ss[w] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = sm[0], S = ss[0];
    for (int i = 1; i < (int)(blockDim.x / 32); ++i) combine(M, S, sm[i], ss[i]);
    const int64_t lab = labels[row];
    const bool ignored = lab == ignore_index;
    const bool valid = !ignored && lab >= 0 && lab < vocab;
    const float tgt = valid ? __bfloat162float(x[lab]) : 0.f;
    // w: 1 = counted, 0 = ignored, -1 = label outside [0, vocab) (the mean becomes NaN)
    rows_out[row] = make_float4(M, S, tgt, valid ? 1.f : (ignored ? 0.f : -1.f));
  }
}

// One block: loss = sum over valid rows of (max + log(sumexp) - target) / #valid.
__global__ void __launch_bounds__(1024) noalloc_mean_kernel(const float4* __restrict__ rows_in,
                                                            int64_t nrows, float* __restrict__ loss_out) {
  float acc = 0.f, cnt = 0.f, bad = 0.f;
  for (int64_t r = threadIdx.x; r < nrows; r += blockDim.x) {
    const float4 st = rows_in[r];
    if (st.w > 0.f) {
      acc += st.x + logf(st.y) - st.z;
      cnt += 1.f;
    } else if (st.w < 0.f) {
      bad += 1.f;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    acc += __shfl_xor_sync(0xffffffff, acc, o);
    cnt += __shfl_xor_sync(0xffffffff, cnt, o);
    bad += __shfl_xor_sync(0xffffffff, bad, o);
  }
  __shared__ float sa[32], sc[32], sb[32];
  const int w = threadIdx.x / 32;
  if ((threadIdx.x & 31) == 0) {
    sa[w] = acc;
    sc[w] = cnt;
    sb[w] = bad;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float A = 0.f, Cn = 0.f, Bd = 0.f;
    for (int i = 0; i < (int)(blockDim.x / 32); ++i) {
      A += sa[i];
      Cn += sc[i];
      Bd += sb[i];
    }
    // NaN when no row is valid (a mean over an empty set) or when a label was out of range
    loss_out[0] = Bd > 0.f ? __int_as_float(0x7fc00000) : A / Cn;
  }
}

// Device address of the scratch array, looked up once per device (with that device current).
constexpr int kMaxDevices = 64;
float4* g_scratch_ptr[kMaxDevices] = {nullptr};
std::mutex g_setup_mutex;

float4* scratch_for_current_device(int* err) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *err = 3;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_xent_noalloc_rows);
    if (e != cudaSuccess || p == nullptr) {
      *err = 3;
      return nullptr;
    }
    g_scratch_ptr[dev] = static_cast<float4*>(p);
  }
  return g_scratch_ptr[dev];
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int ft_xent_mean_loss_noalloc(
    const void* logits, const int64_t* labels, int64_t rows, int64_t vocab, int64_t ld,
    int64_t ignore_index, float* loss_out, void* stream) {
  if (rows > FT_XENT_NOALLOC_MAX_ROWS) return 1;
  // with zero rows neither input is read, so they may be null (an empty tensor's pointer)
  const bool inputs_ok = rows == 0 || (logits != nullptr && labels != nullptr &&
                                       (reinterpret_cast<uintptr_t>(logits) & 15u) == 0);
  if (rows < 0 || !inputs_ok || loss_out == nullptr || vocab <= 0 || vocab % 8 != 0 ||
      ld < vocab || ld % 8 != 0 || vocab > (1ll << 30))
    return 2;
  int err = 0;
  float4* scratch = scratch_for_current_device(&err);
  if (scratch == nullptr) return err;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (rows > 0)
    noalloc_rows_kernel<<<static_cast<unsigned>(rows), 512, 0, st>>>(
        static_cast<const __nv_bfloat16*>(logits), labels, scratch, static_cast<int>(vocab), ld,
        ignore_index);
  noalloc_mean_kernel<<<1, 1024, 0, st>>>(scratch, rows, loss_out);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : 1000 + static_cast<int>(e);
}
