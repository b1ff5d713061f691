/*
 * cuZipNN-B200: C ABI of the B200-native (sm_100a) codec library, libcuzipnn_b200.so.
 *
 * Every entry point takes plain pointers and sizes, works on caller-owned device memory, allocates
 * nothing, enqueues its work on the given CUDA stream (a cudaStream_t passed as void*; NULL is the
 * legacy default stream) on the current device, and returns ZN_OK or a negative status.
 * zn_last_error() describes the last failure of the calling thread.  Calls are reentrant: their
 * state lives in the caller's buffers, with two exceptions: zn_crc32_noalloc's scratch is one
 * static device array that every call on a device shares (see its declaration), and the opt-in
 * kernel timing (zn_timing_*) keeps one process-wide list of events.
 *
 * The reference (ruihe774/cuZipNN) is a Python package whose GPU work goes through two internal
 * seams: Triton kernels (src/cuzipnn/_kernels.py) and ctypes bindings of NVIDIA nvCOMP
 * (src/cuzipnn/_nvcomp.py).  The declarations below name the reference interface each replaces.
 * The whole-tensor entry points (zn_compress, zn_decompress) replace the orchestration of
 * src/cuzipnn/_codec.py with device-side work; the Python package cuzipnn_b200 binds them with
 * ctypes and keeps the reference's public API.
 *
 * Entropy-coded units use this project's ZNR2 rANS payload (nvCOMP's ANS bitstream is closed),
 * and blobs carry version 3 in the header of the reference container (src/cuzipnn/_codec.py:1-21).
 */
#ifndef CUZIPNN_B200_H
#define CUZIPNN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ZN_OK 0
#define ZN_ERR_INVALID (-1) /* bad argument */
#define ZN_ERR_CUDA (-2)    /* a CUDA call or launch failed */
#define ZN_ERR_SPACE (-3)   /* a caller buffer is too small */

#define ZN_ABI_VERSION 1
#define ZN_BLOB_VERSION 3

/* ABI version (ZN_ABI_VERSION). */
int zn_version(void);
/* Message of the calling thread's last failure ("" if none). */
const char *zn_last_error(void);
/* Number of kernels this library has launched in this process (all devices). */
uint64_t zn_launch_count(void);
/* Kernel timing for measurement (no reference counterpart): while enabled, every launch of the
 * named kernel kind ("hist", "encode", "scan", "pack", "dscan", "decode", "decode_overflow",
 * "crc", or "*" for all) is bracketed by CUDA events on its launching stream.  zn_timing_read
 * waits for the recorded events of one kind (NULL: all) and returns the launches' count and the
 * time during which at least one of them ran (the union of their intervals: their summed duration
 * when they do not overlap), then forgets them. */
int zn_timing_enable(const char *kernel, int enable);
int zn_timing_read(const char *kernel, double *total_ms, int64_t *launches);

/* ---- byte-plane seam: replaces src/cuzipnn/_kernels.py:134-188 -------------------------- */

/* split(x, planar, stride, reorder), src/cuzipnn/_kernels.py:134-148: byte b of element e (after
 * the exponent reorder when `reorder`, valid for k = 2 or 4) goes to planar[b * stride + e]. */
int zn_split(const void *x, int64_t n, int k, int reorder, void *planar, int64_t stride, void *stream);

/* merge(src_tbl, base, out, chunk_bytes, reorder), src/cuzipnn/_kernels.py:151-176: stream b of
 * chunk j is read at base + src_tbl[b * nch + j] (int64 byte offsets, device memory). */
int zn_merge(const int64_t *src_tbl, const void *base, void *out, int64_t n, int k, int64_t chunk_bytes,
             int reorder, void *stream);

/* copy_chunks(src_tbl, dst_tbl, nbytes, max_bytes, pad), src/cuzipnn/_kernels.py:179-188: copy
 * nbytes[i] bytes from address src_tbl[i] to dst_tbl[i] (8-byte aligned; tables in device
 * memory); with pad, zero-fill each destination up to a multiple of 8 bytes. */
int zn_copy_chunks(const int64_t *src_tbl, const int64_t *dst_tbl, const int64_t *nbytes, int64_t count,
                   int64_t max_bytes, int pad, void *stream);

/* ---- batched entropy coder: replaces src/cuzipnn/_nvcomp.py:170-257 ---------------------- */

/* max_compressed_chunk_bytes(chunk_bytes, sub_chunks), src/cuzipnn/_nvcomp.py:170-176. */
int64_t zn_ans_max_compressed_chunk_bytes(int64_t chunk_bytes, int sub_chunks);
/* Temp size of zn_ans_compress (nvcompBatchedANSCompressGetTempSizeAsync, _nvcomp.py:198-201). */
size_t zn_ans_compress_temp_bytes(int64_t count, int64_t chunk_bytes, int sub_chunks);
/* compress(...), src/cuzipnn/_nvcomp.py:179-218: ZNR2-encode chunk i (in_bytes[i] <= chunk_bytes
 * bytes at address in_ptrs[i]) into out_ptrs[i]; out_bytes[i] gets its size and statuses[i] 0.
 * sub_chunks is a power of two in [4, 64].  All tables live in device memory. */
int zn_ans_compress(const int64_t *in_ptrs, const int64_t *in_bytes, int64_t chunk_bytes, int64_t count,
                    const int64_t *out_ptrs, int64_t *out_bytes, int32_t *statuses, int sub_chunks,
                    void *temp, size_t temp_bytes, void *stream);
/* Temp size of zn_ans_decompress. */
size_t zn_ans_decompress_temp_bytes(int64_t count);
/* decompress(...), src/cuzipnn/_nvcomp.py:221-257: decode payload i (in_bytes[i] bytes at
 * in_ptrs[i], 8-byte aligned) into out_capacity[i] bytes at out_ptrs[i]; statuses[i] gets 0 or a
 * nonzero error code (the reference allocates but never reads these, _nvcomp.py:241). */
int zn_ans_decompress(const int64_t *in_ptrs, const int64_t *in_bytes, const int64_t *out_capacity,
                      int64_t count, const int64_t *out_ptrs, int32_t *statuses, void *temp, size_t temp_bytes,
                      void *stream);

/* ---- CRC-32: replaces src/cuzipnn/_nvcomp.py:260-287 and src/cuzipnn/_codec.py:116-131 ---- */

size_t zn_crc32_temp_bytes(int64_t nbytes, int64_t segment_bytes);
/* _crc32(data, checksum_chunk_bytes), _codec.py:116-131: out[i] = zlib.crc32 of bytes
 * [i * segment_bytes, min((i + 1) * segment_bytes, nbytes)) of data; any alignment. */
int zn_crc32(const void *data, int64_t nbytes, int64_t segment_bytes, uint32_t *out, void *temp,
             size_t temp_bytes, void *stream);
/* zn_crc32 without the temp buffer.  No counterpart in the reference (there nvCOMP always takes
 * its temp space from torch's allocator).  It is for callers that cannot allocate device memory:
 * a checksum step inside a process whose GPU memory is already owned by another allocator (a
 * serving engine that reserves the free memory up front for weights and KV cache, so that a
 * cudaMalloc fails, and a cudaFree would stall every stream of the device), and C hosts bound
 * through ctypes, cgo or JNI that hold only the device pointers they were handed.  It allocates
 * nothing: its scratch is one fixed 2 MiB array of device memory (524,288 slots, one per 32 KiB
 * block of each segment longer than 32 KiB, e.g. up to 16 GiB of data in segments that are a
 * multiple of 32 KiB), which every GPU that runs it holds until the process exits.  A call that
 * needs more slots returns ZN_ERR_INVALID and launches nothing.  Every call that uses the array
 * looks up its address in the current device's context (so the address stays right after a
 * cudaDeviceReset); the first such call on a device loads the library's device code there, so
 * make it before any stream capture.  All calls on a device share the array: calls whose
 * kernels overlap on the GPU (other streams, or host threads with no ordering between them) race
 * and return wrong CRCs.  Segments of at most 32 KiB do not touch the array. */
int zn_crc32_noalloc(const void *data, int64_t nbytes, int64_t segment_bytes, uint32_t *out, void *stream);

/* ---- whole-tensor codec: replaces src/cuzipnn/_codec.py:308-413 and :471-530 ------------- */

/* Upper bound of the blob size (the size of the `out` buffer zn_compress needs). */
int64_t zn_compress_bound(int64_t n, int k, int ndim, int64_t chunk_bytes);
size_t zn_compress_temp_bytes(int64_t n, int k, int64_t chunk_bytes, int sub_chunks);
/* Compress n elements of k bytes at x (device, 8-byte aligned) into the blob layout of
 * src/cuzipnn/_codec.py:1-21.  `header` (host memory, 24 + 8 * ndim bytes) is the blob header
 * with n_comp left 0; the device fills it in.  The blob goes to out[0, size) and `size` to the
 * device u64 at size_out.  reorder applies to bfloat16 (k = 2) and float32 (k = 4). */
int zn_compress(const void *x, int64_t n, int k, int reorder, const void *header, int header_bytes,
                int64_t chunk_bytes, int sub_chunks, double passthrough_threshold, void *out,
                int64_t out_capacity, uint64_t *size_out, void *temp, size_t temp_bytes, void *stream);

/* Batched form of zn_compress: njobs tensors of the same element size and settings, compressed
 * by one launch per stage (the reference compresses one tensor per call, src/cuzipnn/_codec.py:
 * 231-413).  x, n, headers, header_bytes, out and out_capacity are host arrays with one entry per
 * tensor; sizes_out is a device array of njobs u64. */
size_t zn_compress_batch_temp_bytes(int njobs, const int64_t *n, int k, int64_t chunk_bytes, int sub_chunks);
int zn_compress_batch(int njobs, const void *const *x, const int64_t *n, int k, int reorder,
                      const void *const *headers, const int *header_bytes, int64_t chunk_bytes, int sub_chunks,
                      double passthrough_threshold, void *const *out, const int64_t *out_capacity,
                      uint64_t *sizes_out, void *temp, size_t temp_bytes, void *stream);

size_t zn_decompress_temp_bytes(int64_t n, int k, int64_t chunk_bytes);
/* Decompress the non-stored blob at blob (device, 8-byte aligned, blob_bytes long) whose header
 * fields are given, into out (n * k bytes, device).  n_comp may be -1: the device then reads it
 * from the blob's header, so a caller that knows the other fields needs no host read of the blob.
 * The call sets the device int32 at status: 0, then the OR of the decoding errors; the kernels
 * never read or write out of bounds. */
int zn_decompress(const void *blob, int64_t blob_bytes, int64_t n, int k, int reorder, int ndim,
                  int64_t chunk_bytes, int64_t n_comp, void *out, int32_t *status, void *temp,
                  size_t temp_bytes, void *stream);

/* Batched form of zn_decompress: njobs non-stored blobs of one element size (host arrays, one
 * entry per blob; status is a device array of njobs int32, set as in zn_decompress for every job
 * with n > 0 and left as it is for jobs with n = 0). */
size_t zn_decompress_batch_temp_bytes(int njobs, const int64_t *n, int k, const int64_t *chunk_bytes);
int zn_decompress_batch(int njobs, const void *const *blobs, const int64_t *blob_bytes, const int64_t *n, int k,
                        int reorder, const int *ndim, const int64_t *chunk_bytes, const int64_t *n_comp,
                        void *const *out, int32_t *status, void *temp, size_t temp_bytes, void *stream);

#ifdef __cplusplus
}
#endif

#endif
