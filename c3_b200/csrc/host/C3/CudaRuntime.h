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

// Throws std::runtime_error("<what>: <message>") when rc != 0 (a C3CU_ERR_* status).
void checkAbi(int rc, const char* what);
// Throws on a CUDA runtime error.
void checkCuda(cudaError_t e, const char* what);

}  // namespace cuda
}  // namespace c3
}  // namespace ct
