/* kvc-peer.h — peer-memory result merge for one model compacted on several GPUs.
 *
 * The reference compacts a layer's chunks in one process and merges the chunk
 * results by concatenation in chunk order (src/kv-compact-api.cpp:514-539).
 * When one model's (layer, chunk) units are split across GPUs (one process
 * per GPU), each process writes its slices' results straight into the result
 * arrays of the process that owns the model: the owner allocates them with
 * kvc_peer_alloc, passes the 64-byte handle to the other processes (any
 * channel: a store, a broadcast), and each of them maps it with
 * kvc_peer_open and writes its results there: the batched API's requantised
 * K_out / V_out rows go straight to their place (kvc_layer_result pointers
 * into the mapped buffer), kvc_place_slice merges the kept indices and beta,
 * and kvc_copy_async / kvc_copy2d_async move anything else with the copy
 * engines. Completion is the caller's to order (e.g. a one-element collective
 * on the same streams after the writes).
 *
 * All functions return 0 on success, -1 for a null argument, -12 for a CUDA
 * error and -11 when the allocation fails. The current device of the calling
 * thread is the one used.
 */
#ifndef KVC_PEER_H
#define KVC_PEER_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KVC_PEER_HANDLE_BYTES 64

/* Device memory that other processes can map; *handle receives
 * KVC_PEER_HANDLE_BYTES bytes. */
int kvc_peer_alloc(size_t bytes, void ** ptr, void * handle);
/* Release memory from kvc_peer_alloc (after every mapping of it was closed). */
int kvc_peer_free(void * ptr);
/* Map another process's kvc_peer_alloc memory into this process. */
int kvc_peer_open(const void * handle, void ** ptr);
/* Unmap memory mapped by kvc_peer_open. */
int kvc_peer_close(void * ptr);
/* bytes from src to dst (device or peer-mapped pointers) on `stream`
 * (a cudaStream_t; NULL = the legacy default stream). */
int kvc_copy_async(void * dst, const void * src, size_t bytes, void * stream);
/* height rows of width bytes: row i from src + i*spitch to dst + i*dpitch. */
int kvc_copy2d_async(void * dst, size_t dpitch, const void * src, size_t spitch, size_t width, size_t height,
                     void * stream);

/* Merge one slice's kept indices and beta into a layer's result arrays (local
 * or peer-mapped device memory) on `stream`, with plain stores from one
 * kernel: dst_sel[j] = sel[j] + tok0 (slice-relative indices to layer
 * positions, src/kv-compact-api.cpp:533) and dst_beta[h*beta_ld + j] =
 * beta[h*kept + j] for j < kept, h < H (beta is head-major in both). */
int kvc_place_slice(const int * sel, const float * beta, int kept, int H, int tok0, int * dst_sel,
                    float * dst_beta, int beta_ld, void * stream);

#ifdef __cplusplus
}
#endif

#endif /* KVC_PEER_H */
