// CRC-32 of every segment of a byte buffer, equal to zlib.crc32 (reflected polynomial
// 0x04C11DB7, init and final xor 0xFFFFFFFF).  Replaces nvCOMP's batched CRC32 as used by the
// reference (src/cuzipnn/_nvcomp.py:260-287, src/cuzipnn/_codec.py:116-131).
//
// Method.  The CRC register update is linear over GF(2): after L bytes from initial register I,
// reg = I * x^(8L) mod P  xor  crc0(data), where crc0 is the register for initial value 0, and
// zlib returns ~reg with I = 0xFFFFFFFF.  crc0 of a concatenation A|B is crc0(A) * x^(8|B|) xor
// crc0(B), and leading zero bytes do not change crc0.  So each segment is right-aligned in a
// virtual block of G equal pieces of kPiece bytes (zeros in front); every thread computes crc0 of
// its piece, multiplies it by x^(8 * kPiece * (pieces after it)) from a precomputed table, and an
// XOR reduction gives the block's crc0.  Segments longer than one block (32 KiB) get one thread
// group per block, and a second kernel combines the block values with a binary tree of the
// constant multipliers x^(8 * 32 Ki * 2^k).  The term I * x^(8L) of a segment length L is
// computed on the host.
//
// Lookups.  crc0 of a piece runs slice-by-4 (four 256-entry tables, one lookup per byte).  The
// tables sit in shared memory replicated once per lane (128 KiB, one CTA per SM): lane l reads
// only bank l, so a warp's 32 random lookups take one wavefront instead of ~3.5.  The address of
// a lookup is one byte permute of the data word and the lane's column offset.  Data comes in
// with 32-byte loads, the next 64 bytes in flight while the current ones are hashed; a CTA of 1024
// threads (32 warps) hides the latency of the lookup chains.
#include "zn_common.cuh"

namespace zn {
namespace {

constexpr uint32_t kPoly = 0xEDB88320u;                 // 0x04C11DB7 bit-reflected
constexpr int kPiece = 512;                             // bytes per thread
constexpr int kCrcThreads = 1024;                       // threads per CTA (64 registers each)
constexpr int64_t kBlock = 32768;                       // bytes of one thread group of a long segment
constexpr int kBlockThreads = int(kBlock / kPiece);     // 64: the largest group
constexpr int kTableBytes = 4 * 256 * 32 * 4;           // slice-by-4 tables, one copy per lane
constexpr int kCrcSmem = kTableBytes + kCrcThreads / 32 * 4;
constexpr int kL2Threads = 256;                         // level 2: one CTA per segment

// x^(8 * 2^i) mod P in the reflected representation (bit 31 is x^0), i = 0..63.
struct PowTable {
  uint32_t v[64];
};

constexpr uint32_t gf2_mul_c(uint32_t a, uint32_t b) {
  uint32_t p = 0;
  for (int i = 0; i < 32; ++i) {
    if ((a >> (31 - i)) & 1u) p ^= b;
    b = (b & 1u) ? (b >> 1) ^ kPoly : b >> 1;
  }
  return p;
}

constexpr PowTable make_pow_table() {
  PowTable t{};
  t.v[0] = 0x80000000u >> 8;  // x^8
  for (int i = 1; i < 64; ++i) t.v[i] = gf2_mul_c(t.v[i - 1], t.v[i - 1]);
  return t;
}

__constant__ PowTable c_x8pow = make_pow_table();

// Slice-by-4 tables (t[k][i]: the register after byte i followed by k zero bytes) and the piece
// multipliers x^(8 * kPiece * m) mod P, m < kBlockThreads, computed at compile time.
struct CrcTables {
  uint32_t t[4][256];
  uint32_t piece_pow[kBlockThreads];
};

constexpr CrcTables make_crc_tables() {
  CrcTables r{};
  for (int i = 0; i < 256; ++i) {
    uint32_t c = uint32_t(i);
    for (int b = 0; b < 8; ++b) c = (c >> 1) ^ ((c & 1u) ? kPoly : 0u);
    r.t[0][i] = c;
  }
  for (int i = 0; i < 256; ++i) {
    uint32_t c = r.t[0][i];
    for (int k = 1; k < 4; ++k) {
      c = (c >> 8) ^ r.t[0][c & 0xFF];
      r.t[k][i] = c;
    }
  }
  static_assert(kPiece == 512, "piece_pow uses x^(8 * 2^9)");
  const uint32_t x_piece = make_pow_table().v[9];  // x^(8 * 512)
  r.piece_pow[0] = 0x80000000u;                    // x^0
  for (int m = 1; m < kBlockThreads; ++m) r.piece_pow[m] = gf2_mul_c(r.piece_pow[m - 1], x_piece);
  return r;
}

__device__ const CrcTables g_crc_tables = make_crc_tables();

__device__ __forceinline__ uint32_t gf2_mul(uint32_t a, uint32_t b) {
  uint32_t p = 0;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    p ^= b & (0u - ((a >> (31 - i)) & 1u));
    b = (b >> 1) ^ (kPoly & (0u - (b & 1u)));
  }
  return p;
}

// x^(8 * nbytes) mod P.
__device__ uint32_t x8pow(uint64_t nbytes) {
  uint32_t r = 0;
  for (int i = 0; nbytes; ++i, nbytes >>= 1)
    if (nbytes & 1) r = r ? gf2_mul(r, c_x8pow.v[i]) : c_x8pow.v[i];
  return r ? r : 0x80000000u;  // x^0 = 1
}

// The register term 0xFFFFFFFF * x^(8 L) mod P of a segment of L bytes (host): the CRC of the
// segment is ~(term ^ crc0).
uint32_t init_term(int64_t L) {
  static const PowTable pw = make_pow_table();
  uint32_t r = 0x80000000u;
  for (int i = 0; L; ++i, L >>= 1)
    if (L & 1) r = gf2_mul_c(r, pw.v[i]);
  return gf2_mul_c(0xFFFFFFFFu, r);
}

// ---- shared-memory tables, replicated per lane ------------------------------------------------
// Entry t[k][b] for lane l at byte offset (k >> 1) << 16 | b << 8 | (k & 1) << 7 | l << 2: two
// tables interleave in each 64 KiB half, and a lane's column is fixed, so its bank is l.

__device__ void load_tables(uint8_t* T) {
  for (int i = threadIdx.x; i < kTableBytes / 4; i += blockDim.x) {
    const int k = i >> 13, b = (i >> 5) & 255, l = i & 31;
    *reinterpret_cast<uint32_t*>(T + ((k >> 1) << 16 | b << 8 | (k & 1) << 7 | l << 2)) = g_crc_tables.t[k][b];
  }
  __syncthreads();
}

// t[K][byte POS of x] for the calling lane (lane4 = lane * 4): the byte permute builds
// lane4 | byte << 8, the table's own offset is an immediate.
template <int K, int POS>
__device__ __forceinline__ uint32_t lut(const uint8_t* T, uint32_t x, uint32_t lane4) {
  const uint32_t off = __byte_perm(x, lane4, 0x5504u | (POS << 4));
  return *reinterpret_cast<const uint32_t*>(T + ((K >> 1) << 16) + ((K & 1) << 7) + off);
}

// Four bytes (the little-endian word w) into register c.
__device__ __forceinline__ uint32_t step4(uint32_t c, uint32_t w, const uint8_t* T, uint32_t lane4) {
  const uint32_t x = c ^ w;
  return lut<3, 0>(T, x, lane4) ^ lut<2, 1>(T, x, lane4) ^ lut<1, 2>(T, x, lane4) ^ lut<0, 3>(T, x, lane4);
}

__device__ __forceinline__ uint32_t step1(uint32_t c, uint32_t byte, const uint8_t* T, uint32_t lane4) {
  return lut<0, 0>(T, c ^ byte, lane4) ^ (c >> 8);
}

// 64 bytes from a 32-byte aligned address, as two 32-byte loads.
__device__ __forceinline__ void ld64(const uint8_t* p, uint32_t (&w)[16]) {
#pragma unroll
  for (int q = 0; q < 2; ++q)
    asm volatile("ld.global.nc.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(w[8 * q]), "=r"(w[8 * q + 1]), "=r"(w[8 * q + 2]), "=r"(w[8 * q + 3]), "=r"(w[8 * q + 4]),
                   "=r"(w[8 * q + 5]), "=r"(w[8 * q + 6]), "=r"(w[8 * q + 7])
                 : "l"(p + 32 * q));
}

// crc0 of the len bytes at p (any alignment): bytes up to the next 32-byte boundary, then 64-byte
// chunks (the next chunk's loads issued before the current one is hashed), then 32-byte chunks,
// words and bytes.
__device__ __forceinline__ uint32_t crc_piece(const uint8_t* p, int len, const uint8_t* T, uint32_t lane4) {
  uint32_t c = 0;
  const int head = min(len, int((32 - (reinterpret_cast<uintptr_t>(p) & 31)) & 31));
  for (int i = 0; i < head; ++i) c = step1(c, p[i], T, lane4);
  p += head;
  len -= head;
  const int nch = len >> 6;
  if (nch > 0) {
    uint32_t A[16], B[16];
    ld64(p, A);
    for (int q = 0; q < nch; q += 2) {
      if (q + 1 < nch) ld64(p + 64 * (q + 1), B);
#pragma unroll
      for (int i = 0; i < 16; ++i) c = step4(c, A[i], T, lane4);
      if (q + 1 >= nch) break;
      if (q + 2 < nch) ld64(p + 64 * (q + 2), A);
#pragma unroll
      for (int i = 0; i < 16; ++i) c = step4(c, B[i], T, lane4);
    }
    p += nch << 6;
    len -= nch << 6;
  }
  for (; len >= 32; p += 32, len -= 32) {
    uint32_t w[8];
    asm volatile("ld.global.nc.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]), "=r"(w[4]), "=r"(w[5]), "=r"(w[6]), "=r"(w[7])
                 : "l"(p));
#pragma unroll
    for (int i = 0; i < 8; ++i) c = step4(c, w[i], T, lane4);
  }
  for (; len >= 4; p += 4, len -= 4) c = step4(c, *reinterpret_cast<const uint32_t*>(p), T, lane4);
  for (int i = 0; i < len; ++i) c = step1(c, p[i], T, lane4);
  return c;
}

// Level 1: persistent CTAs (one per SM) over the work items, kCrcThreads / G groups of G threads
// at a time.  single: an item is a segment of at most G * kPiece bytes, whose CRC the group writes
// to out (init_full, init_last: the init terms of a full and of the last segment).  Otherwise an
// item is a 32 KiB block of a long segment (G = kBlockThreads), whose crc0 goes to partial[].
// The loop bound is the same for every thread of the CTA (the group reductions synchronise).
__global__ void __launch_bounds__(kCrcThreads, 1) crc_pieces(const uint8_t* __restrict__ data, int64_t nbytes,
                                                             int64_t seg, int64_t nseg, int G, int64_t bps,
                                                             bool single, uint32_t init_full, uint32_t init_last,
                                                             uint32_t* __restrict__ out, uint32_t* __restrict__ partial) {
  extern __shared__ __align__(16) uint8_t T[];
  uint32_t* red = reinterpret_cast<uint32_t*>(T + kTableBytes);
  load_tables(T);
  const int tid = threadIdx.x, lt = tid % G;
  const uint32_t lane4 = uint32_t(tid & 31) << 2;
  const int gpc = kCrcThreads / G;
  const int64_t items = single ? nseg : nseg * bps;
  // This thread's piece multiplier x^(8 * kPiece * (pieces after it in the group)).
  const uint32_t mult = g_crc_tables.piece_pow[G - 1 - lt];
  for (int64_t base = int64_t(blockIdx.x) * gpc; base < items; base += int64_t(gridDim.x) * gpc) {
    const int64_t it = base + tid / G;
    int64_t s = 0;
    uint32_t c = 0;
    if (it < items) {
      s = single ? it : it / bps;
      const int64_t b = single ? 0 : it % bps;
      const int64_t L = (s == nseg - 1) ? nbytes - s * seg : seg;
      const int64_t nb = single ? 1 : cdiv(L, kBlock);
      const int64_t pad = nb * int64_t(G) * kPiece - L;  // virtual leading zeros
      const int64_t v0 = b * int64_t(G) * kPiece + int64_t(lt) * kPiece;
      const int64_t lo = max(v0 - pad, int64_t(0)), hi = min(v0 + kPiece - pad, L);
      if (hi > lo) c = crc_piece(data + s * seg + lo, int(hi - lo), T, lane4);
      if (c && lt != G - 1) c = gf2_mul(c, mult);
    }
#pragma unroll
    for (int o = 1; o < 32; o <<= 1)
      if (o < G) c ^= __shfl_xor_sync(0xFFFFFFFFu, c, o);
    if (G > 32) {  // groups of whole warps: XOR the warps' values
      if ((tid & 31) == 0) red[tid >> 5] = c;
      __syncthreads();
      if (lt == 0)
        for (int w = 1; w < G / 32; ++w) c ^= red[(tid >> 5) + w];
      __syncthreads();
    }
    if (lt == 0 && it < items) {
      if (single) out[s] = ~((s == nseg - 1 ? init_last : init_full) ^ c);
      else partial[it] = c;
    }
  }
}

// Tree-combine the crc0 values of the kL2Threads threads of a CTA that hold equal pieces of
// `piece_bytes` virtual bytes each; the result ends in thread 0.
__device__ uint32_t combine_group(uint32_t c, uint64_t piece_bytes, uint32_t* sm, uint32_t* mult) {
  const int t = threadIdx.x;
  int levels = 0;
  while ((1 << levels) < kL2Threads) ++levels;
  if (t < levels) mult[t] = x8pow(piece_bytes << t);
  __syncthreads();
  for (int k = 0; k < levels; ++k) {
    const int span = 1 << k;
    sm[t] = c;
    __syncthreads();
    if ((t & (2 * span - 1)) == 0) c = gf2_mul(c, mult[k]) ^ sm[t + span];
    __syncthreads();
  }
  return c;
}

// Level 2: one CTA per segment combines its blocks' crc0 values (right-aligned like level 1).
__global__ void __launch_bounds__(kL2Threads) crc_level2(int64_t nbytes, int64_t seg, int64_t nseg,
                                                         int64_t blocks_per_seg, uint32_t init_full, uint32_t init_last,
                                                         const uint32_t* __restrict__ partial,
                                                         uint32_t* __restrict__ out) {
  __shared__ uint32_t sm[kL2Threads];
  __shared__ uint32_t mult[16];
  __shared__ uint32_t step;
  const int64_t s = blockIdx.x;
  const int t = threadIdx.x;
  const int64_t L = (s == nseg - 1) ? nbytes - s * seg : seg;
  const int64_t nb = cdiv(L, kBlock);
  const int64_t q = cdiv(nb, kL2Threads);  // blocks per thread
  const int64_t shift = q * kL2Threads - nb;
  if (t == 0) step = x8pow(uint64_t(kBlock));
  __syncthreads();
  uint32_t h = 0;
  for (int64_t v = int64_t(t) * q; v < int64_t(t + 1) * q; ++v) {
    const int64_t bi = v - shift;
    if (bi < 0) continue;  // leading virtual zero blocks
    h = (h ? gf2_mul(h, step) : 0u) ^ partial[s * blocks_per_seg + bi];
  }
  h = combine_group(h, uint64_t(q) * kBlock, sm, mult);
  if (t == 0) out[s] = ~((s == nseg - 1 ? init_last : init_full) ^ h);
}

// Both levels for data[0, nbytes) in segments of segment_bytes.  partial: one u32 slot per
// 32 KiB block of every segment longer than 32 KiB (crc_blocks), unused otherwise.
int64_t crc_blocks(int64_t nbytes, int64_t segment_bytes) {
  const int64_t seg = min(segment_bytes, nbytes);  // the longest segment
  return seg > kBlock ? cdiv(nbytes, segment_bytes) * cdiv(seg, kBlock) : 0;
}

int launch_crc(const uint8_t* d, int64_t nbytes, int64_t segment_bytes, uint32_t* out, uint32_t* partial,
               cudaStream_t st, const char* who) {
  const int64_t nseg = cdiv(nbytes, segment_bytes);
  const int64_t seg = min(segment_bytes, nbytes);
  const int64_t bps = seg > kBlock ? cdiv(seg, kBlock) : 0;
  int G = kBlockThreads;
  if (bps == 0) {
    G = 1;
    while (int64_t(G) * kPiece < seg) G <<= 1;
  }
  const int64_t items = bps ? nseg * bps : nseg;
  if (items > 0x7FFFFFFF || nseg > 0x7FFFFFFF) return set_error(ZN_ERR_INVALID, "%s: too many segments", who);
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return set_error(ZN_ERR_CUDA, "%s: %s", who, cudaGetErrorString(e));
  if (int rc = set_max_smem(reinterpret_cast<const void*>(crc_pieces), kCrcSmem)) return rc;
  const int64_t grid = min(int64_t(sms), cdiv(items, int64_t(kCrcThreads / G)));
  const uint32_t init_full = init_term(seg), init_last = init_term(nbytes - (nseg - 1) * segment_bytes);
  {
    TimedLaunch tl("crc", st);
    crc_pieces<<<unsigned(grid), kCrcThreads, kCrcSmem, st>>>(d, nbytes, segment_bytes, nseg, G, bps, bps == 0,
                                                              init_full, init_last, out, partial);
    if (bps) crc_level2<<<unsigned(nseg), kL2Threads, 0, st>>>(nbytes, segment_bytes, nseg, bps, init_full, init_last,
                                                              partial, out);
  }
  count_launch(bps ? 2 : 1);
  return check_launch(who);
}

}  // namespace
}  // namespace zn

using namespace zn;

extern "C" {

size_t zn_crc32_temp_bytes(int64_t nbytes, int64_t segment_bytes) {
  if (nbytes <= 0 || segment_bytes <= 0) return 0;
  return size_t(crc_blocks(nbytes, segment_bytes)) * sizeof(uint32_t);
}

int zn_crc32(const void* data, int64_t nbytes, int64_t segment_bytes, uint32_t* out, void* temp,
             size_t temp_bytes, void* stream) {
  if (nbytes < 0 || segment_bytes <= 0) return set_error(ZN_ERR_INVALID, "zn_crc32: bad arguments");
  if (nbytes == 0) return ZN_OK;
  const int64_t blocks = crc_blocks(nbytes, segment_bytes);
  if (blocks && (!temp || temp_bytes < size_t(blocks) * sizeof(uint32_t)))
    return set_error(ZN_ERR_SPACE, "zn_crc32: temp buffer too small");
  return launch_crc(static_cast<const uint8_t*>(data), nbytes, segment_bytes, out, static_cast<uint32_t*>(temp),
                    static_cast<cudaStream_t>(stream), "zn_crc32");
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// zn_crc32_noalloc: the same kernels with their partial-CRC scratch in a static device array,
// for callers that must not allocate device memory (see the declaration in the public header).
//
// The array is 2 MiB: 524,288 u32 slots, one per 32 KiB block of every segment longer than
// 32 KiB.  Each GPU that runs this code holds it until the process exits.  All calls on a device
// share it and it keeps the previous call's contents; every slot a call reads is written earlier
// in the same call (level 1 writes all nseg * blocks_per_seg slots before level 2 reads them, in
// stream order), so nothing needs clearing.  Two calls whose kernels overlap on the GPU (different
// streams, or host threads with no ordering between them) race on the array.

namespace {

constexpr int64_t kNoAllocSlots = int64_t(1) << 19;  // 2 MiB of u32

}  // namespace

static __device__ __align__(256) uint32_t g_crc_noalloc_scratch[kNoAllocSlots];

namespace {

// Device address of the scratch array in the current device's context.  Looked up on every call
// (a cheap query once the module is loaded): a cached address would go stale after a
// cudaDeviceReset, which gives the device a new context.  The first lookup on a device loads the
// library's device code there.
int noalloc_scratch(uint32_t** ptr) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_crc_noalloc_scratch);
  if (e != cudaSuccess || !p)
    return set_error(ZN_ERR_CUDA, "zn_crc32_noalloc: cudaGetSymbolAddress of the scratch array: %s",
                     cudaGetErrorString(e));
  *ptr = static_cast<uint32_t*>(p);
  return ZN_OK;
}

}  // namespace

extern "C" int zn_crc32_noalloc(const void* data, int64_t nbytes, int64_t segment_bytes, uint32_t* out,
                                void* stream) {
  if (nbytes < 0 || segment_bytes <= 0) return set_error(ZN_ERR_INVALID, "zn_crc32_noalloc: bad arguments");
  if (nbytes == 0) return ZN_OK;
  const int64_t slots = crc_blocks(nbytes, segment_bytes);
  if (slots > kNoAllocSlots)
    return set_error(ZN_ERR_INVALID,
                     "zn_crc32_noalloc: %lld bytes in segments of %lld need %lld scratch slots (one per 32 KiB block "
                     "of each segment); the static scratch holds %lld (2 MiB). Use zn_crc32 with a temp buffer",
                     (long long)nbytes, (long long)segment_bytes, (long long)slots, (long long)kNoAllocSlots);
  uint32_t* partial = nullptr;  // segments of at most 32 KiB: the scratch is neither touched nor looked up
  if (slots)
    if (int rc = noalloc_scratch(&partial)) return rc;
  return launch_crc(static_cast<const uint8_t*>(data), nbytes, segment_bytes, out, partial,
                    static_cast<cudaStream_t>(stream), "zn_crc32_noalloc");
}
