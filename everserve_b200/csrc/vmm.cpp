// Driver VMM calls through the runtime's entry-point query (the extension does not link libcuda).
#include "vmm.h"

#include <cuda.h>
#include <cuda_runtime.h>
#include <unistd.h>

#include <mutex>

namespace es {
namespace vmm {
namespace {

struct Api {
  decltype(&cuMemCreate) create = nullptr;
  decltype(&cuMemRelease) release = nullptr;
  decltype(&cuMemAddressReserve) reserve = nullptr;
  decltype(&cuMemAddressFree) free_range = nullptr;
  decltype(&cuMemMap) map = nullptr;
  decltype(&cuMemUnmap) unmap = nullptr;
  decltype(&cuMemSetAccess) access = nullptr;
  decltype(&cuMemGetAllocationGranularity) granularity = nullptr;
  decltype(&cuMemExportToShareableHandle) export_handle = nullptr;
  decltype(&cuMemImportFromShareableHandle) import_handle = nullptr;
  bool ok = false;
};

template <typename F>
void get(const char* name, F& fn, bool& ok) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
    p = nullptr;
  fn = reinterpret_cast<F>(p);
  ok = ok && p != nullptr;
}

const Api& api() {
  static Api a;
  static std::once_flag once;
  std::call_once(once, [] {
    bool ok = true;
    get("cuMemCreate", a.create, ok);
    get("cuMemRelease", a.release, ok);
    get("cuMemAddressReserve", a.reserve, ok);
    get("cuMemAddressFree", a.free_range, ok);
    get("cuMemMap", a.map, ok);
    get("cuMemUnmap", a.unmap, ok);
    get("cuMemSetAccess", a.access, ok);
    get("cuMemGetAllocationGranularity", a.granularity, ok);
    get("cuMemExportToShareableHandle", a.export_handle, ok);
    get("cuMemImportFromShareableHandle", a.import_handle, ok);
    a.ok = ok;
  });
  return a;
}

CUmemAllocationProp prop_for(int device) {
  CUmemAllocationProp p = {};
  p.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  p.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  p.location.id = device;
  p.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  return p;
}

bool map_range(const Api& a, int device, CUmemGenericAllocationHandle h, uint64_t size, Buffer& out,
               const char** err) {
  CUdeviceptr va = 0;
  if (a.reserve(&va, size, 0, 0, 0) != CUDA_SUCCESS) {
    *err = "cuMemAddressReserve failed";
    return false;
  }
  if (a.map(va, size, 0, h, 0) != CUDA_SUCCESS) {
    a.free_range(va, size);
    *err = "cuMemMap failed";
    return false;
  }
  CUmemAccessDesc acc = {};
  acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  acc.location.id = device;
  acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  if (a.access(va, size, &acc, 1) != CUDA_SUCCESS) {
    a.unmap(va, size);
    a.free_range(va, size);
    *err = "cuMemSetAccess failed (no peer access between these devices?)";
    return false;
  }
  out.ptr = va;
  out.size = size;
  out.handle = h;
  return true;
}

}  // namespace

uint64_t rounded(int device, uint64_t bytes) {
  const Api& a = api();
  if (!a.ok) return bytes;
  CUmemAllocationProp p = prop_for(device);
  size_t g = 0;
  if (a.granularity(&g, &p, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED) != CUDA_SUCCESS || g == 0) g = 2 << 20;
  return (bytes + g - 1) / g * g;
}

bool create(int device, uint64_t bytes, Buffer& out, const char** err) {
  const Api& a = api();
  if (!a.ok) {
    *err = "the driver has no VMM entry points";
    return false;
  }
  cudaFree(nullptr);  // a context on the current device
  const uint64_t size = rounded(device, bytes);
  CUmemAllocationProp p = prop_for(device);
  CUmemGenericAllocationHandle h = 0;
  if (a.create(&h, size, &p, 0) != CUDA_SUCCESS) {
    *err = "cuMemCreate failed";
    return false;
  }
  if (!map_range(a, device, h, size, out, err)) {
    a.release(h);
    return false;
  }
  int fd = -1;
  if (a.export_handle(&fd, h, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0) != CUDA_SUCCESS) {
    release(out);
    *err = "cuMemExportToShareableHandle failed";
    return false;
  }
  out.fd = fd;
  return true;
}

bool import(int device, int fd, uint64_t bytes, Buffer& out, const char** err) {
  const Api& a = api();
  if (!a.ok) {
    *err = "the driver has no VMM entry points";
    return false;
  }
  cudaFree(nullptr);
  CUmemGenericAllocationHandle h = 0;
  if (a.import_handle(&h, reinterpret_cast<void*>(static_cast<intptr_t>(fd)),
                      CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR) != CUDA_SUCCESS) {
    *err = "cuMemImportFromShareableHandle failed";
    return false;
  }
  if (!map_range(a, device, h, rounded(device, bytes), out, err)) {
    a.release(h);
    return false;
  }
  out.fd = -1;
  return true;
}

void release(Buffer& b) {
  const Api& a = api();
  if (!a.ok || b.ptr == 0) return;
  a.unmap(b.ptr, b.size);
  a.free_range(b.ptr, b.size);
  a.release(b.handle);
  if (b.fd >= 0) ::close(b.fd);
  b = Buffer{};
}

}  // namespace vmm
}  // namespace es
