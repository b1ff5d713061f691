/*
 * CPU oracle for the cuZipNN codec path.  TEST INFRASTRUCTURE ONLY: the product (the
 * cuzipnn_b200 package and its CUDA library) never links, loads or calls this code.  Only the
 * tests, the smoke check and the CPU baseline of the benchmark use it, and only as the checker.
 *
 * What it restates, from the reference (ruihe774/cuZipNN, paths relative to that project):
 *   - bit reorder / revert         src/cuzipnn/_kernels.py:17-31
 *   - byte split into planes       src/cuzipnn/_kernels.py:34-54, :134-148
 *   - byte merge out of planes     src/cuzipnn/_kernels.py:57-105, :151-176
 *   - batched chunk copy           src/cuzipnn/_kernels.py:108-131, :179-188
 *   - sub-chunk count              src/cuzipnn/_codec.py:83-86
 *   - passthrough rule and blob    src/cuzipnn/_codec.py:74-80, :89-93, :270-306, :361-403
 *   - blob parse and decompress    src/cuzipnn/_codec.py:416-542
 *   - CRC-32 as zlib.crc32         src/cuzipnn/_codec.py:116-131 (nvCOMP CRC32 spec at
 *                                  src/cuzipnn/_nvcomp.py:75-76: poly 0x04C11DB7, reflected,
 *                                  init and xorout 0xFFFFFFFF)
 *
 * The reference's entropy coder is nvCOMP's batched ANS (nvidia-libnvcomp-cu13 5.3.0.16, a
 * closed binary; call sites src/cuzipnn/_nvcomp.py:179-257).  Its bitstream is not public, so
 * this project defines its own payload format, "ZNR2", built from the published rANS method
 * (J. Duda, "Asymmetric numeral systems", 2013; F. Giesen, "Interleaved entropy coders", 2014),
 * and this file is the normative statement of that format:
 *
 *   Scale: 12 bits (M = 4096).  State: u32 in [L, 2^31) with L = 2^15.  I/O: 16-bit words.
 *   Coding symbol s (frequency f, cumulative frequency cum) maps x to
 *   (x / f) * M + x % f + cum; before that, a state with x >= f * 2^19 writes its low 16 bits
 *   to its stream and shifts right by 16.  The encoder starts every state at L.
 *   A plane chunk of m symbols (1 <= m <= 2^24) is cut into sub-chunks of
 *   sc = roundup(ceil(m / n_sub), 128) symbols; nu = ceil(m / sc) of them are non-empty.
 *   Each sub-chunk is coded by 8 interleaved states ("lanes"), each with its own word stream.
 *   Round r, step i (0..15), lane l (0..7) covers symbol r*128 + l*16 + i of the sub-chunk
 *   when that index is below the sub-chunk length.  The decoder runs rounds and steps forward;
 *   a lane decodes its symbol and, if its state fell below L, reads the next word of its own
 *   stream.  The encoder runs the same schedule backwards (last step first), so each stream is
 *   stored in the reverse of the order its words were produced.
 *
 *   Frequencies: counts c[s]; np = number of present symbols; smax = most frequent symbol
 *   (lowest index on ties).  np == 1: f[smax] = M.  Otherwise f[s] = max(1, (c*M + m/2) / m)
 *   for present symbols; d = M - sum f; if f[smax] + d >= 1 then f[smax] += d, else
 *   f[s] = 1 + c*(M - np) / m for present symbols and f[smax] absorbs the remainder.
 *
 *   Payload (little-endian):
 *     [0]      u8  log2(n_sub), 2..6
 *     [1]      u8  0
 *     [2,34)   presence bitmap, bit (s & 7) of byte (s >> 3)
 *     [34,..)  f[s] - 1 as 12-bit fields for present symbols in ascending order,
 *              field k at bits [12k, 12k+12), zero-padded to a 4-byte boundary
 *     lengths  nu * 8 stream lengths in words (sub-chunk-major, then lane), u16 if
 *              sc / 8 < 65536 else u32, padded to 4 bytes
 *     states   nu * 8 u32 final encoder states (the decoder's initial states), same order
 *     streams  the nu * 8 word streams back to back, same order
 */
#ifndef ZN_ORACLE_H
#define ZN_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ZN_ORC_BLOB_VERSION 3

/* Exponent bit reorder for W = 16 (bfloat16) or W = 32 (float32). */
uint64_t orc_reorder(uint64_t u, int w);
uint64_t orc_revert(uint64_t u, int w);

/* planar[b * stride + e] = byte b of (reordered) element e. */
void orc_split(const uint8_t *x, int64_t n, int k, int reorder, uint8_t *planar, int64_t stride);

/* out[e] = revert(OR_b src_b[e] << 8b); stream b of chunk j starts at base + src_tbl[b*nch + j]. */
void orc_merge(const int64_t *src_tbl, const uint8_t *base, uint8_t *out, int64_t n, int k,
               int64_t chunk_bytes, int reorder);

/* Copy nbytes[i] bytes from src_base + src_off[i] to dst_base + dst_off[i]; with pad, zero-fill
 * the destination up to the next multiple of 8. */
void orc_copy_chunks(const uint8_t *src_base, const int64_t *src_off, uint8_t *dst_base,
                     const int64_t *dst_off, const int64_t *nbytes, int64_t count, int pad);

/* zlib.crc32(data, crc). */
uint32_t orc_crc32(uint32_t crc, const uint8_t *p, int64_t n);
/* CRC-32 of each seg-byte segment (the last one may be shorter). */
void orc_crc32_segments(const uint8_t *p, int64_t n, int64_t seg, uint32_t *out);

int orc_sub_chunks(int64_t chunk_bytes, int64_t sub_chunk_bytes);

/* Frequency normalisation of the ZNR2 format (exposed for tests). */
void orc_normalize(const uint32_t counts[256], int64_t m, uint32_t freqs[256]);

int64_t orc_ans_max_payload(int64_t m, int n_sub);
/* Encode m symbols; returns the payload size, or -1 if cap is too small. */
int64_t orc_ans_encode(const uint8_t *sym, int64_t m, int n_sub, uint8_t *out, int64_t cap);
/* Decode a payload of `size` bytes into m symbols; 0 on success, else a negative error. */
int orc_ans_decode(const uint8_t *payload, int64_t size, int64_t m, uint8_t *out);

/* Worst-case blob size of the non-stored layout. */
int64_t orc_blob_bound(int64_t n, int k, int ndim, int64_t chunk_bytes);

/* The whole compressor (stored path included).  Returns the blob size or a negative error. */
int64_t orc_compress(const uint8_t *x, int64_t n, int k, int dtype_code, int reorder, int ndim,
                     const int64_t *shape, int64_t chunk_bytes, int n_sub, double threshold,
                     int64_t min_compress_bytes, int version, uint8_t *out, int64_t cap,
                     int threads);

/* Decompress a blob into out (n * k bytes).  Returns 0 or a negative error. */
int orc_decompress(const uint8_t *blob, int64_t size, uint8_t *out, int64_t out_bytes,
                   int version, int threads);

#ifdef __cplusplus
}
#endif

#endif
