// Device plumbing of the C3 B200 host layer: the stream the CUDA kernel objects launch
// on, and stream-ordered device allocation from CUDA's default memory pool (kept cached:
// the pool's release threshold is raised so freed blocks are reused, not returned).
#pragma once

#include <cuda_runtime_api.h>

#include <cstddef>
#include <string>

namespace ct {
namespace c3 {
namespace cuda {

// Stream used by every CUDA CompiledKernel of the calling thread (default: legacy stream 0).
cudaStream_t currentStream();
void setCurrentStream(cudaStream_t s);

// True when a CUDA device is usable from this process.
bool deviceAvailable();

// Stream-ordered allocation on the current device and the calling thread's current stream;
// throws std::runtime_error on failure. freeDevice returns the block on `stream`, the stream it
// was allocated on: work on other streams must be ordered before the release by the host (as
// with any stream-ordered allocator), and the stream must outlive the block.
void* allocDevice(size_t bytes);
void freeDevice(void* p, cudaStream_t stream);

// Copies between pageable host memory (a host framework's tensors) and device memory on
// `stream`. Large copies go through the library's pinned staging buffers in chunks: a pool of
// host threads copies one chunk between the host tensor and a staging buffer while the DMA of
// the neighbouring chunk runs, so the link moves pinned-speed transfers although the host
// tensor itself is not pinned. copyToDevice returns once `src` may be reused (the last DMA may
// still be in flight on `stream`); copyToHost returns once `dst` holds the data. Small copies
// (under 4 MiB) are plain cudaMemcpyAsync calls. Each device has its own staging buffers (the
// current device's are used, so `stream` and the device buffer belong to the current device);
// large copies from different host threads to one device are serialised on them.
void copyToDevice(void* dst, const void* src, size_t bytes, cudaStream_t stream);
void copyToHost(void* dst, const void* src, size_t bytes, cudaStream_t stream);

// Throws std::runtime_error("<what>: <message>") when rc != 0 (a C3CU_ERR_* status).
void checkAbi(int rc, const char* what);
// Throws on a CUDA runtime error.
void checkCuda(cudaError_t e, const char* what);

}  // namespace cuda
}  // namespace c3
}  // namespace ct
