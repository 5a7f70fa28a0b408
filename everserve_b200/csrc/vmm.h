// Device memory shared between processes with the driver's virtual memory management (VMM).
//
// A buffer is a physical allocation (cuMemCreate, exportable as a POSIX file descriptor) mapped at
// a reserved virtual range with read/write access for the owning device. Another process imports
// the descriptor (passed over a Unix socket), maps it at its own range and grants its own device
// access (a peer mapping over NVLink). The physical memory lives until every mapping and every
// handle is released, in every process: a member that dies leaves its buffer valid for the
// survivors that mapped it, so a collective that is still writing to (or reading from) a dead
// member touches live memory and only waits out its bound. (Legacy CUDA IPC does not give this:
// an exporter that exits frees the memory under its importers.)
#pragma once

#include <cstdint>

namespace es {
namespace vmm {

struct Buffer {
  uint64_t ptr = 0;    // device virtual address
  uint64_t size = 0;   // bytes (a multiple of the allocation granularity)
  uint64_t handle = 0; // CUmemGenericAllocationHandle
  int fd = -1;         // exported POSIX descriptor (creator only; -1 for imports)
};

// Granularity-rounded size of an allocation of `bytes` on `device`.
uint64_t rounded(int device, uint64_t bytes);
// Create, map and zero nothing: returns false and a message on failure.
bool create(int device, uint64_t bytes, Buffer& out, const char** err);
// Import a descriptor another process exported; maps it with access for `device`.
bool import(int device, int fd, uint64_t bytes, Buffer& out, const char** err);
// Unmap, free the range and release the handle (closes the exported descriptor, if any).
void release(Buffer& b);

}  // namespace vmm
}  // namespace es
