// SM-driven peer transfers of the fused tensor-parallel collectives (sequence parallelism).
//
// All-gather -> GEMM: every rank stages its token shard in a symmetric slot and publishes a
// READY flag to its peers.  ag_pull_kernel (a few CTAs on a side stream, one per SM the gated
// GEMM leaves free) visits the ranks in ring order starting with itself; for each it waits
// (bounded) for the owner's READY flag, copies the owner's chunk over NVLink into the local
// gathered buffer with 16-byte loads (many in flight per thread), and each CTA then adds 1 to
// the chunk's local counter (release).  The GEMM's TMA producer waits per tile until the
// counter of every chunk its rows touch reaches epoch x CTAs, so the MMAs on the local chunk
// start at once and the peers' rows are consumed as they land; each remote row crosses
// NVLink once.
//
// GEMM -> reduce-scatter: every rank's GEMM stores its full partial output [T, N] into its
// own symmetric slot (local stores) and publishes PART.  rs_pull_kernel, on the owner of
// token rows [me*Tl, (me+1)*Tl), waits (bounded) for every peer's PART flag and sums those
// rows of every peer's slot in fp32 (P2P loads), adds the residual and writes bf16.
//
// Every wait gives up after its time limit, records an error code in the device status word
// and returns; nothing here spins without a bound.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <vector>

#include "common.cuh"

namespace ft {

constexpr int TP_MAX_RANKS = 8;
constexpr int AG_UNROLL = 8;

struct AGPullArgs {
  const uint4* src[TP_MAX_RANKS];   // every rank's staged chunk (peer addresses)
  const int* ready[TP_MAX_RANKS];   // this rank's READY flag of each owner (local)
  uint4* dst;                       // gathered buffer, world x chunk_vec
  int* chunk_count;                 // local counters [world]
  int64_t chunk_vec;                // 16-byte vectors per chunk
  int world, me, epoch;
  int* err;
  uint64_t timeout_ns;
};

__device__ __forceinline__ uint64_t tp_now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait by one thread: *flag - value >= 0.  Records code on timeout.
__device__ __forceinline__ bool tp_wait_geq(const int* flag, int value, int* err, int code,
                                            uint64_t timeout_ns) {
  const uint64_t t0 = tp_now_ns();
  uint32_t backoff = 32;
  while (true) {
    int v;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    if (v - value >= 0) return true;
    if (tp_now_ns() - t0 > timeout_ns) {
      atomicCAS(err, 0, code);
      return false;
    }
    __nanosleep(backoff);
    if (backoff < 1024) backoff <<= 1;
  }
}

__global__ void __launch_bounds__(1024, 1) ag_pull_kernel(const __grid_constant__ AGPullArgs a) {
  __shared__ int ok;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int k = 0; k < a.world; ++k) {
    const int r = (a.me + k) % a.world;
    if (threadIdx.x == 0)
      ok = (r == a.me) ? 1 : (tp_wait_geq(a.ready[r], a.epoch, a.err, 200 + r, a.timeout_ns) ? 1 : 0);
    __syncthreads();
    if (!ok) return;   // the gated GEMM then times out on this chunk and records its own code
    const uint4* __restrict__ s = a.src[r];
    uint4* __restrict__ d = a.dst + static_cast<int64_t>(r) * a.chunk_vec;
    int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    // AG_UNROLL independent 16-byte peer loads in flight per thread, then the stores
    for (; i + (AG_UNROLL - 1) * stride < a.chunk_vec; i += AG_UNROLL * stride) {
      uint4 v[AG_UNROLL];
#pragma unroll
      for (int u = 0; u < AG_UNROLL; ++u) v[u] = s[i + u * stride];
#pragma unroll
      for (int u = 0; u < AG_UNROLL; ++u) d[i + u * stride] = v[u];
    }
    for (; i < a.chunk_vec; i += stride) d[i] = s[i];
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      asm volatile("red.release.gpu.global.add.s32 [%0], 1;" ::"l"(a.chunk_count + r) : "memory");
    }
  }
}

struct RSPullArgs {
  const uint4* src[TP_MAX_RANKS];   // every rank's partial rows for this owner (peer addresses)
  const int* part[TP_MAX_RANKS];    // this rank's PART flag of each peer (local)
  const uint4* resid;               // optional residual rows (local)
  uint4* out;                       // this rank's reduced rows (local)
  int64_t nvec;
  int world, epoch;
  int* err;
  uint64_t timeout_ns;
};

__global__ void __launch_bounds__(256) rs_pull_kernel(const __grid_constant__ RSPullArgs a) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    int good = 1;
    for (int r = 0; r < a.world && good; ++r)
      good = tp_wait_geq(a.part[r], a.epoch, a.err, 240 + r, a.timeout_ns) ? 1 : 0;
    ok = good;
  }
  __syncthreads();
  if (!ok) return;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < a.nvec;
       v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    uint4 q[TP_MAX_RANKS];
#pragma unroll
    for (int r = 0; r < TP_MAX_RANKS; ++r)
      if (r < a.world) q[r] = a.src[r][v];
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
    for (int r = 0; r < TP_MAX_RANKS; ++r) {
      if (r >= a.world) break;
      const uint32_t w[4] = {q[r].x, q[r].y, q[r].z, q[r].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = unpack_bf16x2(w[j]);
        acc[2 * j] += f.x;
        acc[2 * j + 1] += f.y;
      }
    }
    if (a.resid) {
      const uint4 rq = a.resid[v];
      const uint32_t w[4] = {rq.x, rq.y, rq.z, rq.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = unpack_bf16x2(w[j]);
        acc[2 * j] += f.x;
        acc[2 * j + 1] += f.y;
      }
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    a.out[v] = o;
  }
}

namespace {
void check_aligned(int64_t p, const char* what) {
  TORCH_CHECK((p & 15) == 0, what, " must be 16-byte aligned");
}
}  // namespace

// Gather `world` chunks of `chunk_bytes` (peer addresses src_ptrs[r]) into dst (local, world x
// chunk_bytes) with `ctas` CTAs on the current stream; see ag_pull_kernel.
void ag_pull(const std::vector<int64_t>& src_ptrs, const std::vector<int64_t>& ready_ptrs,
             torch::Tensor& dst, int64_t chunk_bytes, int64_t chunk_count_ptr, int64_t me,
             int64_t epoch, int64_t ctas, torch::Tensor& err, int64_t timeout_ms) {
  const int world = static_cast<int>(src_ptrs.size());
  TORCH_CHECK(world >= 1 && world <= TP_MAX_RANKS && static_cast<int>(ready_ptrs.size()) == world,
              "ag_pull: 1..8 ranks");
  TORCH_CHECK(chunk_bytes % 16 == 0 && dst.is_contiguous() && dst.numel() * dst.element_size() >= world * chunk_bytes,
              "ag_pull: chunk must be a multiple of 16 bytes and dst large enough");
  TORCH_CHECK(me >= 0 && me < world && ctas >= 1 && ctas <= 1024 && timeout_ms > 0);
  AGPullArgs a{};
  for (int r = 0; r < world; ++r) {
    check_aligned(src_ptrs[r], "ag_pull source");
    a.src[r] = reinterpret_cast<const uint4*>(src_ptrs[r]);
    a.ready[r] = reinterpret_cast<const int*>(ready_ptrs[r]);
  }
  check_aligned(reinterpret_cast<int64_t>(dst.data_ptr()), "ag_pull destination");
  a.dst = reinterpret_cast<uint4*>(dst.data_ptr());
  a.chunk_count = reinterpret_cast<int*>(chunk_count_ptr);
  a.chunk_vec = chunk_bytes / 16;
  a.world = world;
  a.me = static_cast<int>(me);
  a.epoch = static_cast<int>(epoch);
  a.err = err.data_ptr<int>();
  a.timeout_ns = static_cast<uint64_t>(timeout_ms) * 1000000ull;
  const c10::cuda::CUDAGuard g(dst.device());
  ag_pull_kernel<<<static_cast<unsigned>(ctas), 1024, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// out[i] = sum_r src_r[i] (+ resid[i]) over `nelem` bf16 elements, after every PART flag
// reached `epoch`; see rs_pull_kernel.
void rs_pull(const std::vector<int64_t>& src_ptrs, const std::vector<int64_t>& part_ptrs,
             const c10::optional<torch::Tensor>& resid, torch::Tensor& out, int64_t nelem,
             int64_t epoch, torch::Tensor& err, int64_t timeout_ms) {
  const int world = static_cast<int>(src_ptrs.size());
  TORCH_CHECK(world >= 1 && world <= TP_MAX_RANKS && static_cast<int>(part_ptrs.size()) == world,
              "rs_pull: 1..8 ranks");
  TORCH_CHECK(nelem % 8 == 0 && out.scalar_type() == at::kBFloat16 && out.is_contiguous() &&
              out.numel() >= nelem, "rs_pull: bf16 output of >= nelem elements, nelem % 8 == 0");
  TORCH_CHECK(timeout_ms > 0);
  RSPullArgs a{};
  for (int r = 0; r < world; ++r) {
    check_aligned(src_ptrs[r], "rs_pull source");
    a.src[r] = reinterpret_cast<const uint4*>(src_ptrs[r]);
    a.part[r] = reinterpret_cast<const int*>(part_ptrs[r]);
  }
  if (resid.has_value()) {
    TORCH_CHECK(resid->scalar_type() == at::kBFloat16 && resid->is_contiguous() && resid->numel() >= nelem);
    check_aligned(reinterpret_cast<int64_t>(resid->data_ptr()), "rs_pull residual");
    a.resid = reinterpret_cast<const uint4*>(resid->data_ptr());
  }
  check_aligned(reinterpret_cast<int64_t>(out.data_ptr()), "rs_pull output");
  a.out = reinterpret_cast<uint4*>(out.data_ptr());
  a.nvec = nelem / 8;
  a.world = world;
  a.epoch = static_cast<int>(epoch);
  a.err = err.data_ptr<int>();
  a.timeout_ns = static_cast<uint64_t>(timeout_ms) * 1000000ull;
  const c10::cuda::CUDAGuard g(out.device());
  int dev, sms;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((a.nvec + 255) / 256, 4 * sms)));
  rs_pull_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace ft
