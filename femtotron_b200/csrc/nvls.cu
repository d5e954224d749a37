// NVLink SHARP (NVLS) multicast buffers and the in-switch all-reduce built on them.
//
// A multicast object groups one physical allocation per GPU of a process group; loads and
// stores through its multicast address are executed by the NVSwitch on every member's copy:
// `multimem.ld_reduce` returns the sum over all members' values of an address and
// `multimem.st` writes a value into every member's copy.  Each process
//   1. creates (rank 0) or imports (the others, from a POSIX file descriptor that the Python
//      side passes over a Unix socket) the multicast object,
//   2. adds its device to the team,
//   3. creates its physical allocation (shareable, as imported multicast objects require),
//      binds it to the object and maps it twice: a unicast address (its own copy) and the
//      multicast address,
//   4. tears everything down in the reverse order in nvls_close.
// All checks of sizes and device support run before anything is bound.
//
// All-reduce of n elements resident in every rank's unicast copy (two-shot, in the switch):
//   barrier -> each rank reduces its 1/world slice with multimem.ld_reduce (fp32 accumulation
//   for bf16) and writes the result back to every member with multimem.st -> barrier.
// The barrier is one thread: multimem.red.release adds 1 to a counter in every member's copy,
// then it waits (bounded) until its own copy reaches epoch x world.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda.h>

#include <map>
#include <mutex>
#include <stdexcept>
#include <string>

#include "common.cuh"

namespace ft {

namespace {

template <typename F>
F drv(const char* name) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || p == nullptr)
    throw std::runtime_error(std::string("femtotron_b200 nvls: driver entry point missing: ") + name);
  return reinterpret_cast<F>(p);
}

void ck(CUresult r, const char* what) {
  if (r != CUDA_SUCCESS)
    throw std::runtime_error(std::string("femtotron_b200 nvls: ") + what + " failed, CUresult " +
                             std::to_string(static_cast<int>(r)));
}

struct Api {
  decltype(&cuDeviceGet) deviceGet = drv<decltype(&cuDeviceGet)>("cuDeviceGet");
  decltype(&cuDeviceGetAttribute) deviceGetAttribute =
      drv<decltype(&cuDeviceGetAttribute)>("cuDeviceGetAttribute");
  decltype(&cuMulticastCreate) mcCreate = drv<decltype(&cuMulticastCreate)>("cuMulticastCreate");
  decltype(&cuMulticastAddDevice) mcAddDevice = drv<decltype(&cuMulticastAddDevice)>("cuMulticastAddDevice");
  decltype(&cuMulticastBindMem) mcBindMem = drv<decltype(&cuMulticastBindMem)>("cuMulticastBindMem");
  decltype(&cuMulticastUnbind) mcUnbind = drv<decltype(&cuMulticastUnbind)>("cuMulticastUnbind");
  decltype(&cuMulticastGetGranularity) mcGran =
      drv<decltype(&cuMulticastGetGranularity)>("cuMulticastGetGranularity");
  decltype(&cuMemCreate) memCreate = drv<decltype(&cuMemCreate)>("cuMemCreate");
  decltype(&cuMemRelease) memRelease = drv<decltype(&cuMemRelease)>("cuMemRelease");
  decltype(&cuMemAddressReserve) addrReserve = drv<decltype(&cuMemAddressReserve)>("cuMemAddressReserve");
  decltype(&cuMemAddressFree) addrFree = drv<decltype(&cuMemAddressFree)>("cuMemAddressFree");
  decltype(&cuMemMap) memMap = drv<decltype(&cuMemMap)>("cuMemMap");
  decltype(&cuMemUnmap) memUnmap = drv<decltype(&cuMemUnmap)>("cuMemUnmap");
  decltype(&cuMemSetAccess) setAccess = drv<decltype(&cuMemSetAccess)>("cuMemSetAccess");
  decltype(&cuMemGetAllocationGranularity) memGran =
      drv<decltype(&cuMemGetAllocationGranularity)>("cuMemGetAllocationGranularity");
  decltype(&cuMemExportToShareableHandle) exportHandle =
      drv<decltype(&cuMemExportToShareableHandle)>("cuMemExportToShareableHandle");
  decltype(&cuMemImportFromShareableHandle) importHandle =
      drv<decltype(&cuMemImportFromShareableHandle)>("cuMemImportFromShareableHandle");
};

Api& api() {
  static Api a;
  return a;
}

struct Nvls {
  int device = 0;
  int world = 0;
  size_t size = 0;
  CUmemGenericAllocationHandle mc = 0, phys = 0;
  CUdeviceptr uc_va = 0, mc_va = 0;
  bool added = false, bound = false, uc_mapped = false, mc_mapped = false;
};

std::mutex g_mu;
std::map<int64_t, Nvls> g_nvls;
int64_t g_next = 1;

CUmulticastObjectProp mc_prop(int world, size_t size) {
  CUmulticastObjectProp p{};
  p.numDevices = static_cast<unsigned>(world);
  p.size = size;
  p.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  return p;
}

CUmemAllocationProp phys_prop(int device) {
  CUmemAllocationProp p{};
  p.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  p.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  p.location.id = device;
  p.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  return p;
}

Nvls& get(int64_t id) {
  auto it = g_nvls.find(id);
  TORCH_CHECK(it != g_nvls.end(), "nvls: unknown handle ", id);
  return it->second;
}

}  // namespace

// True when `device` supports multicast objects (NVLS).
bool nvls_supported(int64_t device) {
  CUdevice d;
  if (api().deviceGet(&d, static_cast<int>(device)) != CUDA_SUCCESS) return false;
  int v = 0;
  if (api().deviceGetAttribute(&v, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, d) != CUDA_SUCCESS) return false;
  return v != 0;
}

// `nbytes` rounded up to the granularity both the multicast object and the physical
// allocation need.
int64_t nvls_round_size(int64_t device, int64_t world, int64_t nbytes) {
  CUmulticastObjectProp mp = mc_prop(static_cast<int>(world), static_cast<size_t>(nbytes));
  size_t g1 = 0, g2 = 0;
  ck(api().mcGran(&g1, &mp, CU_MULTICAST_GRANULARITY_RECOMMENDED), "cuMulticastGetGranularity");
  CUmemAllocationProp pp = phys_prop(static_cast<int>(device));
  ck(api().memGran(&g2, &pp, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED), "cuMemGetAllocationGranularity");
  size_t g = std::max(g1, g2);
  return static_cast<int64_t>((static_cast<size_t>(nbytes) + g - 1) / g * g);
}

// Rank 0: create the multicast object.  Returns a handle id; nvls_export_fd gives the file
// descriptor to pass to the peers.
int64_t nvls_create(int64_t device, int64_t world, int64_t size) {
  TORCH_CHECK(nvls_supported(device), "nvls: device does not support multicast");
  const c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  Nvls n;
  n.device = static_cast<int>(device);
  n.world = static_cast<int>(world);
  n.size = static_cast<size_t>(size);
  CUmulticastObjectProp mp = mc_prop(n.world, n.size);
  ck(api().mcCreate(&n.mc, &mp), "cuMulticastCreate");
  std::lock_guard<std::mutex> l(g_mu);
  g_nvls[g_next] = n;
  return g_next++;
}

int64_t nvls_export_fd(int64_t id) {
  std::lock_guard<std::mutex> l(g_mu);
  Nvls& n = get(id);
  int fd = -1;
  ck(api().exportHandle(&fd, n.mc, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0),
     "cuMemExportToShareableHandle");
  return fd;
}

// The other ranks: import the multicast object from a file descriptor received from rank 0.
int64_t nvls_import(int64_t device, int64_t world, int64_t size, int64_t fd) {
  TORCH_CHECK(nvls_supported(device), "nvls: device does not support multicast");
  const c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  Nvls n;
  n.device = static_cast<int>(device);
  n.world = static_cast<int>(world);
  n.size = static_cast<size_t>(size);
  ck(api().importHandle(&n.mc, reinterpret_cast<void*>(static_cast<uintptr_t>(fd)),
                        CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR),
     "cuMemImportFromShareableHandle");
  std::lock_guard<std::mutex> l(g_mu);
  g_nvls[g_next] = n;
  return g_next++;
}

void nvls_add_device(int64_t id) {
  std::lock_guard<std::mutex> l(g_mu);
  Nvls& n = get(id);
  CUdevice d;
  ck(api().deviceGet(&d, n.device), "cuDeviceGet");
  ck(api().mcAddDevice(n.mc, d), "cuMulticastAddDevice");
  n.added = true;
}

// Allocate this rank's copy, bind it and map the unicast and multicast addresses.
// Returns (unicast address, multicast address).
std::vector<int64_t> nvls_bind_map(int64_t id) {
  std::lock_guard<std::mutex> l(g_mu);
  Nvls& n = get(id);
  TORCH_CHECK(n.added, "nvls: add the device first");
  const c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(n.device));
  CUmemAllocationProp pp = phys_prop(n.device);
  ck(api().memCreate(&n.phys, n.size, &pp, 0), "cuMemCreate");
  ck(api().mcBindMem(n.mc, 0, n.phys, 0, n.size, 0), "cuMulticastBindMem");
  n.bound = true;
  CUmemAccessDesc acc{};
  acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  acc.location.id = n.device;
  acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  ck(api().addrReserve(&n.uc_va, n.size, 0, 0, 0), "cuMemAddressReserve");
  ck(api().memMap(n.uc_va, n.size, 0, n.phys, 0), "cuMemMap (unicast)");
  n.uc_mapped = true;
  ck(api().setAccess(n.uc_va, n.size, &acc, 1), "cuMemSetAccess (unicast)");
  ck(api().addrReserve(&n.mc_va, n.size, 0, 0, 0), "cuMemAddressReserve");
  ck(api().memMap(n.mc_va, n.size, 0, n.mc, 0), "cuMemMap (multicast)");
  n.mc_mapped = true;
  ck(api().setAccess(n.mc_va, n.size, &acc, 1), "cuMemSetAccess (multicast)");
  TORCH_CHECK(cudaMemset(reinterpret_cast<void*>(n.uc_va), 0, n.size) == cudaSuccess,
              "nvls: clearing the new buffer failed");
  return {static_cast<int64_t>(n.uc_va), static_cast<int64_t>(n.mc_va)};
}

// Tear down in the reverse order (the caller synchronises the device and the group first).
void nvls_close(int64_t id) {
  std::lock_guard<std::mutex> l(g_mu);
  auto it = g_nvls.find(id);
  if (it == g_nvls.end()) return;
  Nvls& n = it->second;
  const c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(n.device));
  cudaDeviceSynchronize();
  if (n.mc_mapped) api().memUnmap(n.mc_va, n.size);
  if (n.mc_va) api().addrFree(n.mc_va, n.size);
  if (n.uc_mapped) api().memUnmap(n.uc_va, n.size);
  if (n.uc_va) api().addrFree(n.uc_va, n.size);
  if (n.bound) {
    CUdevice d;
    if (api().deviceGet(&d, n.device) == CUDA_SUCCESS) api().mcUnbind(n.mc, d, 0, n.size);
  }
  if (n.phys) api().memRelease(n.phys);
  if (n.mc) api().memRelease(n.mc);
  g_nvls.erase(it);
}

// ------------------------------------------------------------------------------------------
// kernels
// ------------------------------------------------------------------------------------------
__global__ void nvls_barrier_kernel(unsigned* mc_flag, const unsigned* uc_flag, unsigned target,
                                    int* err, int code, uint64_t timeout_ns) {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  asm volatile("multimem.red.release.sys.global.add.u32 [%0], 1;" ::"l"(mc_flag) : "memory");
  uint64_t t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  uint32_t backoff = 32;
  while (true) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(uc_flag) : "memory");
    if (static_cast<int>(v - target) >= 0) return;
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (t - t0 > timeout_ns) {
      atomicCAS(err, 0, code);
      return;
    }
    __nanosleep(backoff);
    if (backoff < 1024) backoff <<= 1;
  }
}

constexpr int NVLS_UNROLL = 4;

template <bool F32>
__device__ __forceinline__ void nvls_ld_reduce(const uint4* p, uint32_t (&r)[4]) {
  if (F32)
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "l"(p) : "memory");
  else
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "l"(p) : "memory");
}

template <bool F32>
__device__ __forceinline__ void nvls_st(uint4* p, uint32_t (&r)[4], float scale) {
  if (scale != 1.f) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (F32) {
        r[j] = __float_as_uint(__uint_as_float(r[j]) * scale);
      } else {
        const float2 f = unpack_bf16x2(r[j]);
        r[j] = pack_bf16x2(f.x * scale, f.y * scale);
      }
    }
  }
  if (F32)
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};"
                 ::"l"(p), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]) : "memory");
  else
    asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1, %2, %3, %4};"
                 ::"l"(p), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]) : "memory");
}

// This rank's slice [v0, v1) of 16-byte vectors: NVLS_UNROLL in-switch reductions in flight per
// thread, then the broadcast stores of their results.
template <bool F32>
__global__ void __launch_bounds__(256) nvls_reduce_kernel(uint4* mc, int64_t v0, int64_t v1, float scale) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  int64_t v = v0 + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  for (; v + (NVLS_UNROLL - 1) * stride < v1; v += NVLS_UNROLL * stride) {
    uint32_t r[NVLS_UNROLL][4];
#pragma unroll
    for (int u = 0; u < NVLS_UNROLL; ++u) nvls_ld_reduce<F32>(mc + v + u * stride, r[u]);
#pragma unroll
    for (int u = 0; u < NVLS_UNROLL; ++u) nvls_st<F32>(mc + v + u * stride, r[u], scale);
  }
  for (; v < v1; v += stride) {
    uint32_t r[4];
    nvls_ld_reduce<F32>(mc + v, r);
    nvls_st<F32>(mc + v, r, scale);
  }
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}

// One NVLS barrier on the current stream: counter at byte `flag_off` of the buffer; `target`
// = (number of barriers so far, this one included) x world.
void nvls_barrier(int64_t uc_base, int64_t mc_base, int64_t flag_off, int64_t target,
                  torch::Tensor& err, int64_t code, int64_t timeout_ms) {
  TORCH_CHECK((flag_off & 3) == 0 && timeout_ms > 0);
  nvls_barrier_kernel<<<1, 1, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<unsigned*>(mc_base + flag_off), reinterpret_cast<const unsigned*>(uc_base + flag_off),
      static_cast<unsigned>(target), err.data_ptr<int>(), static_cast<int>(code),
      static_cast<uint64_t>(timeout_ms) * 1000000ull);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// In-switch reduction of this rank's slice of `nbytes` at the start of the buffer (every
// rank's unicast copy holds its contribution; afterwards every copy holds the result of the
// slice).  f32 or bf16 (fp32 accumulation); `scale` multiplies the sum (1/world: average).
void nvls_reduce_slice(int64_t mc_base, int64_t nbytes, int64_t rank, int64_t world, bool f32,
                       double scale) {
  TORCH_CHECK(nbytes % 16 == 0 && (mc_base & 15) == 0, "nvls: 16-byte aligned sizes");
  const int64_t nvec = nbytes / 16;
  const int64_t per = (nvec + world - 1) / world;
  const int64_t v0 = std::min(nvec, rank * per), v1 = std::min(nvec, v0 + per);
  if (v1 <= v0) return;
  int dev, sms;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((v1 - v0 + 255) / 256, 4 * sms)));
  auto st = at::cuda::getCurrentCUDAStream();
  uint4* mc = reinterpret_cast<uint4*>(mc_base);
  if (f32)
    nvls_reduce_kernel<true><<<grid, 256, 0, st>>>(mc, v0, v1, static_cast<float>(scale));
  else
    nvls_reduce_kernel<false><<<grid, 256, 0, st>>>(mc, v0, v1, static_cast<float>(scale));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace ft
