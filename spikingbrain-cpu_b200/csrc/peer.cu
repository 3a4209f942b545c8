// Peer memory for output-channel shards on several GPUs of one node: one arena per rank, exported
// and mapped with CUDA IPC so that every rank can store into (and signal) every other rank's
// buffers over NVLink.  The kernels that use the mappings are in gemv.cu.
#include <cstring>

#include "common.cuh"

using namespace sbq;

static_assert(sizeof(cudaIpcMemHandle_t) == SBQ_PEER_HANDLE_BYTES, "IPC handle size");

extern "C" int sbq_peer_alloc(size_t bytes, void** ptr) {
    if (!ptr || bytes == 0) return set_error(SBQ_ERR_INVALID_ARGUMENT, "null pointer or zero size");
    *ptr = nullptr;
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) return set_error(SBQ_ERR_CUDA, "peer arena of %zu bytes: %s", bytes, cudaGetErrorString(e));
    e = cudaMemset(p, 0, bytes);
    if (e != cudaSuccess) {
        cudaFree(p);
        return set_error(SBQ_ERR_CUDA, "clear peer arena: %s", cudaGetErrorString(e));
    }
    *ptr = p;
    return SBQ_OK;
}

extern "C" int sbq_peer_free(void* ptr) {
    if (!ptr) return SBQ_OK;
    cudaError_t e = cudaFree(ptr);
    return e == cudaSuccess ? SBQ_OK : set_error(SBQ_ERR_CUDA, "free peer arena: %s", cudaGetErrorString(e));
}

extern "C" int sbq_peer_handle(const void* ptr, void* handle) {
    if (!ptr || !handle) return set_error(SBQ_ERR_INVALID_ARGUMENT, "null pointer");
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
    if (e != cudaSuccess) return set_error(SBQ_ERR_CUDA, "export peer arena: %s", cudaGetErrorString(e));
    std::memcpy(handle, &h, sizeof(h));
    return SBQ_OK;
}

extern "C" int sbq_peer_open(const void* handle, void** ptr) {
    if (!handle || !ptr) return set_error(SBQ_ERR_INVALID_ARGUMENT, "null pointer");
    *ptr = nullptr;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return set_error(SBQ_ERR_CUDA, "map peer arena: %s", cudaGetErrorString(e));
    *ptr = p;
    return SBQ_OK;
}

extern "C" int sbq_peer_close(void* ptr) {
    if (!ptr) return SBQ_OK;
    cudaError_t e = cudaIpcCloseMemHandle(ptr);
    return e == cudaSuccess ? SBQ_OK : set_error(SBQ_ERR_CUDA, "unmap peer arena: %s", cudaGetErrorString(e));
}
