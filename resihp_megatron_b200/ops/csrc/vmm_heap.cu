// Symmetric-heap regions from the CUDA virtual memory management API (cuMem*), shared between the
// processes of one node as POSIX file descriptors.
//
// An exporter creates a physical allocation on its GPU, maps it into a reserved virtual range and
// exports a file descriptor; an importer turns the descriptor back into an allocation handle and
// maps it into its own reserved range with read/write access for its own GPU (peer access over
// NVLink).  Unlike a cudaIpc mapping, an imported handle holds a reference on the physical memory:
// when the exporting process dies, the survivors' mappings of its region stay valid until they
// unmap them, so a late load from a departed peer reads stale data instead of faulting.
//
// Driver entry points come from cudaGetDriverEntryPoint (no link-time dependency on libcuda).
// Every function returns 0 or a CUDA driver / runtime error code; none throws.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <unordered_map>

#include "kernels.h"

namespace rb {
namespace {

struct Api {
  decltype(&cuMemGetAllocationGranularity) granularity = nullptr;
  decltype(&cuMemCreate) create = nullptr;
  decltype(&cuMemAddressReserve) reserve = nullptr;
  decltype(&cuMemMap) map = nullptr;
  decltype(&cuMemSetAccess) set_access = nullptr;
  decltype(&cuMemExportToShareableHandle) export_handle = nullptr;
  decltype(&cuMemImportFromShareableHandle) import_handle = nullptr;
  decltype(&cuMemUnmap) unmap = nullptr;
  decltype(&cuMemAddressFree) address_free = nullptr;
  decltype(&cuMemRelease) release = nullptr;
  bool ok = false;
};

template <class F>
bool entry(const char* name, F& fn) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
    return false;
  fn = reinterpret_cast<F>(p);
  return true;
}

const Api& api() {
  static Api a;
  static std::once_flag once;
  std::call_once(once, [] {
    a.ok = entry("cuMemGetAllocationGranularity", a.granularity) && entry("cuMemCreate", a.create) &&
           entry("cuMemAddressReserve", a.reserve) && entry("cuMemMap", a.map) &&
           entry("cuMemSetAccess", a.set_access) && entry("cuMemExportToShareableHandle", a.export_handle) &&
           entry("cuMemImportFromShareableHandle", a.import_handle) && entry("cuMemUnmap", a.unmap) &&
           entry("cuMemAddressFree", a.address_free) && entry("cuMemRelease", a.release);
  });
  return a;
}

struct Mapping {
  CUmemGenericAllocationHandle handle;
  size_t size;
};

std::mutex g_mu;
std::unordered_map<uintptr_t, Mapping>& mappings() {
  static auto* m = new std::unordered_map<uintptr_t, Mapping>();  // never destroyed (process exit)
  return *m;
}

CUmemAllocationProp device_prop(int device) {
  CUmemAllocationProp prop = {};
  prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  prop.location.id = device;
  prop.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  return prop;
}

// Reserve a range, map `h` into it and give `device` read/write access; undoes itself on failure.
int map_handle(CUmemGenericAllocationHandle h, size_t size, size_t align, int device, void** ptr) {
  const Api& a = api();
  CUdeviceptr va = 0;
  CUresult r = a.reserve(&va, size, align, 0, 0);
  if (r != CUDA_SUCCESS) return static_cast<int>(r);
  r = a.map(va, size, 0, h, 0);
  if (r != CUDA_SUCCESS) {
    a.address_free(va, size);
    return static_cast<int>(r);
  }
  CUmemAccessDesc acc = {};
  acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  acc.location.id = device;
  acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  r = a.set_access(va, size, &acc, 1);
  if (r != CUDA_SUCCESS) {
    a.unmap(va, size);
    a.address_free(va, size);
    return static_cast<int>(r);
  }
  *ptr = reinterpret_cast<void*>(va);
  std::lock_guard<std::mutex> lock(g_mu);
  mappings()[static_cast<uintptr_t>(va)] = Mapping{h, size};
  return 0;
}

size_t granularity_of(int device) {
  const CUmemAllocationProp prop = device_prop(device);
  size_t g = 0;
  if (api().granularity(&g, &prop, CU_MEM_ALLOC_GRANULARITY_MINIMUM) != CUDA_SUCCESS || g == 0) g = 2u << 20;
  return g;
}

}  // namespace

int vmm_available() { return api().ok ? 1 : 0; }

long long vmm_round(int device, long long bytes) {
  if (!api().ok) return -1;
  const long long g = static_cast<long long>(granularity_of(device));
  return (bytes + g - 1) / g * g;
}

int vmm_alloc(int device, long long bytes, void** ptr, int* fd) {
  const Api& a = api();
  if (!a.ok) return -1;
  if (bytes <= 0) return -2;
  if (cudaSetDevice(device) != cudaSuccess) return -3;
  const CUmemAllocationProp prop = device_prop(device);
  const size_t g = granularity_of(device);
  const size_t size = (static_cast<size_t>(bytes) + g - 1) / g * g;
  CUmemGenericAllocationHandle h;
  CUresult r = a.create(&h, size, &prop, 0);
  if (r != CUDA_SUCCESS) return static_cast<int>(r);
  int shareable = -1;
  r = a.export_handle(&shareable, h, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0);
  if (r != CUDA_SUCCESS) {
    a.release(h);
    return static_cast<int>(r);
  }
  const int rc = map_handle(h, size, g, device, ptr);
  if (rc != 0) {
    a.release(h);
    return rc;
  }
  *fd = shareable;
  return 0;
}

int vmm_import(int device, int fd, long long bytes, void** ptr) {
  const Api& a = api();
  if (!a.ok) return -1;
  if (bytes <= 0 || fd < 0) return -2;
  if (cudaSetDevice(device) != cudaSuccess) return -3;
  CUmemGenericAllocationHandle h;
  CUresult r = a.import_handle(&h, reinterpret_cast<void*>(static_cast<uintptr_t>(fd)),
                               CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR);
  if (r != CUDA_SUCCESS) return static_cast<int>(r);
  const int rc = map_handle(h, static_cast<size_t>(bytes), granularity_of(device), device, ptr);
  if (rc != 0) a.release(h);
  return rc;
}

int vmm_free(void* ptr) {
  const Api& a = api();
  if (!a.ok) return -1;
  Mapping m;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    auto it = mappings().find(reinterpret_cast<uintptr_t>(ptr));
    if (it == mappings().end()) return -2;
    m = it->second;
    mappings().erase(it);
  }
  const CUdeviceptr va = reinterpret_cast<CUdeviceptr>(ptr);
  CUresult r = a.unmap(va, m.size);
  const CUresult r2 = a.address_free(va, m.size);
  const CUresult r3 = a.release(m.handle);
  if (r == CUDA_SUCCESS) r = r2 != CUDA_SUCCESS ? r2 : r3;
  return static_cast<int>(r);
}

}  // namespace rb
