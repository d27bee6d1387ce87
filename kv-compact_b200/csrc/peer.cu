// peer.cu — result merge across processes through CUDA IPC (include/kvc-peer.h).
// The owner of a model's result arrays allocates them here and exports an IPC
// handle; the processes that computed other slices map it and write their
// results into it over NVLink: the requantisation kernels store K_out / V_out
// rows there directly, k_place_slice stores the kept indices (offset to
// layer positions) and the head-major beta runs, and copy-engine copies
// (cudaMemcpyAsync / cudaMemcpy2DAsync) are there for anything else. All of
// it is plain stores or copies: no receive is posted on the owner, which
// keeps computing while the results land.
#include "kvc_internal.h"
#include "kvc-peer.h"

#include <cuda_runtime.h>

static_assert(sizeof(cudaIpcMemHandle_t) <= KVC_PEER_HANDLE_BYTES, "IPC handle larger than the public buffer");

namespace {
// blockIdx.y < H: beta row h; blockIdx.y == H: the indices.
__global__ void __launch_bounds__(256) k_place_slice(const int * __restrict__ sel, const float * __restrict__ beta,
                                                     int kept, int H, int tok0, int * __restrict__ dst_sel,
                                                     float * __restrict__ dst_beta, int beta_ld) {
    const int j = blockIdx.x * 256 + threadIdx.x;
    if (j >= kept) return;
    const int h = blockIdx.y;
    if (h == H) dst_sel[j] = sel[j] + tok0;
    else dst_beta[(size_t)h * beta_ld + j] = beta[(size_t)h * kept + j];
}
}  // namespace

extern "C" {

KVC_EXPORT int kvc_peer_alloc(size_t bytes, void ** ptr, void * handle) {
    if (!ptr || !handle || bytes == 0) return KVC_ERR_NULL;
    *ptr = nullptr;
    void * p = nullptr;
    KVC_CUDA(cudaMalloc(&p, bytes));
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        fprintf(stderr, "[kvc] cudaIpcGetMemHandle: %s\n", cudaGetErrorString(e));
        cudaFree(p);
        return KVC_ERR_CUDA;
    }
    memset(handle, 0, KVC_PEER_HANDLE_BYTES);
    memcpy(handle, &h, sizeof(h));
    *ptr = p;
    return KVC_OK;
}

KVC_EXPORT int kvc_peer_free(void * ptr) {
    if (!ptr) return KVC_ERR_NULL;
    KVC_CUDA(cudaFree(ptr));
    return KVC_OK;
}

KVC_EXPORT int kvc_peer_open(const void * handle, void ** ptr) {
    if (!handle || !ptr) return KVC_ERR_NULL;
    *ptr = nullptr;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void * p = nullptr;
    KVC_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
    *ptr = p;
    return KVC_OK;
}

KVC_EXPORT int kvc_peer_close(void * ptr) {
    if (!ptr) return KVC_ERR_NULL;
    KVC_CUDA(cudaIpcCloseMemHandle(ptr));
    return KVC_OK;
}

KVC_EXPORT int kvc_copy_async(void * dst, const void * src, size_t bytes, void * stream) {
    if (bytes == 0) return KVC_OK;
    if (!dst || !src) return KVC_ERR_NULL;
    KVC_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, (cudaStream_t)stream));
    return KVC_OK;
}

KVC_EXPORT int kvc_copy2d_async(void * dst, size_t dpitch, const void * src, size_t spitch, size_t width,
                                size_t height, void * stream) {
    if (width == 0 || height == 0) return KVC_OK;
    if (!dst || !src) return KVC_ERR_NULL;
    KVC_CUDA(cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, height, cudaMemcpyDefault, (cudaStream_t)stream));
    return KVC_OK;
}

KVC_EXPORT int kvc_place_slice(const int * sel, const float * beta, int kept, int H, int tok0, int * dst_sel,
                               float * dst_beta, int beta_ld, void * stream) {
    if (kept == 0) return KVC_OK;
    if (!sel || !beta || !dst_sel || !dst_beta) return KVC_ERR_NULL;
    if (kept < 0 || H <= 0 || H > 65535 || beta_ld < kept) return KVC_ERR_DIMS;
    k_place_slice<<<dim3((kept + 255) / 256, H + 1), 256, 0, (cudaStream_t)stream>>>(sel, beta, kept, H, tok0, dst_sel,
                                                                                     dst_beta, beta_ld);
    KVC_CUDA(cudaGetLastError());
    return KVC_OK;
}

}  // extern "C"
