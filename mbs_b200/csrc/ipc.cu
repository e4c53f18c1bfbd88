// Peer-memory plumbing for the N-sharded layer's output exchange.
//
// One rank's output block is pushed into every peer's copy of the gathered
// output with copy-engine transfers over NVLink (cudaMemcpyAsync between
// device pointers of different GPUs, one call per contiguous block), so the
// exchange runs beside the GEMM without taking any of its SMs.  The peers'
// buffers are reached through CUDA IPC handles of buffers this library
// allocates itself (an exact allocation base, so a handle needs no offset).
#include "common.h"

#include <cstring>

using namespace mbs;

extern "C" int mbs_ipc_alloc(size_t bytes, void** ptr, void* handle_out)
{
    clear_error();
    if (ptr == nullptr || handle_out == nullptr || bytes == 0)
        return fail(MBS_ERR_INVALID_ARGUMENT, "mbs_ipc_alloc: null pointer or zero size");
    *ptr = nullptr;
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc (ipc buffer)");
    cudaIpcMemHandle_t h;
    e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess)
    {
        cudaFree(p);
        return cuda_fail(e, "cudaIpcGetMemHandle");
    }
    std::memcpy(handle_out, &h, sizeof(h));
    *ptr = p;
    return MBS_OK;
}

extern "C" int mbs_ipc_open(const void* handle, void** peer_ptr)
{
    clear_error();
    if (handle == nullptr || peer_ptr == nullptr)
        return fail(MBS_ERR_INVALID_ARGUMENT, "mbs_ipc_open: null pointer");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    cudaError_t e = cudaIpcOpenMemHandle(peer_ptr, h, cudaIpcMemLazyEnablePeerAccess);
    return e == cudaSuccess ? MBS_OK : cuda_fail(e, "cudaIpcOpenMemHandle");
}

extern "C" int mbs_ipc_close(void* peer_ptr)
{
    clear_error();
    cudaError_t e = cudaIpcCloseMemHandle(peer_ptr);
    return e == cudaSuccess ? MBS_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

extern "C" int mbs_ipc_free(void* ptr)
{
    clear_error();
    cudaError_t e = cudaFree(ptr);
    return e == cudaSuccess ? MBS_OK : cuda_fail(e, "cudaFree (ipc buffer)");
}

extern "C" int mbs_copy_async(void* dst, const void* src, size_t bytes, void* stream)
{
    clear_error();
    if (bytes == 0) return MBS_OK;
    if (dst == nullptr || src == nullptr) return fail(MBS_ERR_INVALID_ARGUMENT, "mbs_copy_async: null pointer");
    cudaError_t e =
        cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MBS_OK : cuda_fail(e, "cudaMemcpyAsync (peer copy)");
}
