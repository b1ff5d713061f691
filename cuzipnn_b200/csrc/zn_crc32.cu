// CRC-32 of every segment of a byte buffer, equal to zlib.crc32 (reflected polynomial
// 0x04C11DB7, init and final xor 0xFFFFFFFF).  Replaces nvCOMP's batched CRC32 as used by the
// reference (src/cuzipnn/_nvcomp.py:260-287, src/cuzipnn/_codec.py:116-131).
//
// Method.  The CRC register update is linear over GF(2): after L bytes from initial register I,
// reg = I * x^(8L) mod P  xor  crc0(data), where crc0 is the register for initial value 0, and
// zlib returns ~reg with I = 0xFFFFFFFF.  crc0 of a concatenation A|B is crc0(A) * x^(8|B|) xor
// crc0(B), and leading zero bytes do not change crc0.  So each segment is right-aligned in a
// virtual block of G equal pieces (zeros in front), every thread computes crc0 of its 128-byte
// piece with slice-by-8 tables held in shared memory, multiplies it by x^(8 * 128 * (pieces after
// it)) from a precomputed table, and an XOR reduction gives the block's crc0.  Segments longer
// than one block (32 KiB) get one CTA per block and a second kernel combines the block values with
// a binary tree of the constant multipliers x^(8 * 32 Ki * 2^k).
#include "zn_common.cuh"

namespace zn {
namespace {

constexpr uint32_t kPoly = 0xEDB88320u;  // 0x04C11DB7 bit-reflected
constexpr int kPiece = 128;              // bytes per thread
constexpr int kThreads = 256;
constexpr int64_t kBlock = int64_t(kPiece) * kThreads;  // 32 KiB

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

// Slice-by-8 tables (T[k][i]: the register after byte i followed by k zero bytes) and the piece
// multipliers x^(8 * kPiece * m) mod P, m = 0 .. kThreads - 1, computed at compile time.
struct CrcTables {
  uint32_t t[8][256];
  uint32_t piece_pow[256];
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
    for (int k = 1; k < 8; ++k) {
      c = (c >> 8) ^ r.t[0][c & 0xFF];
      r.t[k][i] = c;
    }
  }
  const uint32_t x_piece = make_pow_table().v[7];  // x^(8 * 128)
  static_assert(kPiece == 128, "piece_pow assumes 128-byte pieces");
  r.piece_pow[0] = 0x80000000u;  // x^0
  for (int m = 1; m < 256; ++m) r.piece_pow[m] = gf2_mul_c(r.piece_pow[m - 1], x_piece);
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

__device__ __forceinline__ uint32_t finish(uint32_t crc0, int64_t len) {
  return ~(gf2_mul(0xFFFFFFFFu, x8pow(uint64_t(len))) ^ crc0);
}

// Slice-by-8 tables into shared memory, from the precomputed copy.
__device__ void build_tables(uint32_t (*T)[256]) {
  for (int i = threadIdx.x; i < 8 * 256; i += blockDim.x) T[i >> 8][i & 255] = g_crc_tables.t[i >> 8][i & 255];
  __syncthreads();
}

__device__ __forceinline__ uint32_t crc_bytes(uint32_t c, const uint8_t* p, int64_t n, const uint32_t (*T)[256]) {
  for (int64_t i = 0; i < n; ++i) c = T[0][(c ^ p[i]) & 0xFF] ^ (c >> 8);
  return c;
}

__device__ __forceinline__ uint32_t crc_8(uint32_t c, uint32_t lo, uint32_t hi, const uint32_t (*T)[256]) {
  lo ^= c;
  return T[7][lo & 0xFF] ^ T[6][(lo >> 8) & 0xFF] ^ T[5][(lo >> 16) & 0xFF] ^ T[4][lo >> 24] ^
         T[3][hi & 0xFF] ^ T[2][(hi >> 8) & 0xFF] ^ T[1][(hi >> 16) & 0xFF] ^ T[0][hi >> 24];
}

// crc0 of data[lo, hi) (hi - lo <= kPiece).
__device__ __forceinline__ uint32_t crc_piece(const uint8_t* data, int64_t lo, int64_t hi, const uint32_t (*T)[256]) {
  const uint8_t* p = data + lo;
  if (hi - lo == kPiece && (reinterpret_cast<uintptr_t>(p) & 15) == 0) {
    uint32_t c = 0;
#pragma unroll
    for (int i = 0; i < kPiece; i += 16) {
      const uint4 v = *reinterpret_cast<const uint4*>(p + i);
      c = crc_8(c, v.x, v.y, T);
      c = crc_8(c, v.z, v.w, T);
    }
    return c;
  }
  return hi > lo ? crc_bytes(0, p, hi - lo, T) : 0u;
}

// Tree-combine the crc0 values of G consecutive threads (G a power of two, <= blockDim.x) that
// hold equal pieces of `piece_bytes` virtual bytes each; the group's crc0 ends in its first thread.
// `mult` (shared, >= 9 entries) receives the per-level multipliers x^(8 * piece_bytes * 2^k).
__device__ uint32_t combine_group(uint32_t c, int G, uint64_t piece_bytes, uint32_t* sm, uint32_t* mult) {
  const int t = threadIdx.x;
  int levels = 0;
  while ((1 << levels) < G) ++levels;
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

// Level 1.  Segments of at most kBlock bytes: groups of G threads, one segment per group
// (single_level), writing the final CRC.  Longer segments: one CTA per (segment, block) writing
// the block's crc0 to partial[].
__global__ void __launch_bounds__(kThreads) crc_level1(const uint8_t* __restrict__ data, int64_t nbytes, int64_t seg,
                                                       int64_t nseg, int G, int64_t blocks_per_seg, bool single_level,
                                                       uint32_t* __restrict__ out, uint32_t* __restrict__ partial) {
  __shared__ uint32_t T[8][256];
  __shared__ uint32_t sm[kThreads / 32];
  build_tables(T);
  const int t = threadIdx.x;
  int64_t s, b;
  int lt;  // thread index within its group
  if (single_level) {
    const int groups = kThreads / G;
    s = int64_t(blockIdx.x) * groups + t / G;
    b = 0;
    lt = t % G;
  } else {
    s = blockIdx.x / blocks_per_seg;
    b = blockIdx.x % blocks_per_seg;
    lt = t;
  }
  uint32_t c = 0;
  int64_t L = 0;
  if (s < nseg) {
    L = (s == nseg - 1) ? nbytes - s * seg : seg;
    const int64_t nb = single_level ? 1 : cdiv(L, kBlock);
    const int64_t vlen = nb * int64_t(G) * kPiece;  // virtual (right-aligned) segment length
    const int64_t pad = vlen - L;
    const int64_t v0 = b * int64_t(G) * kPiece + int64_t(lt) * kPiece;
    const int64_t lo = max(v0 - pad, int64_t(0)), hi = min(v0 + kPiece - pad, L);
    if (hi > lo) c = crc_piece(data + s * seg, lo, hi, T);
  }
  // The group's crc0 is the XOR over its pieces of crc0 * x^(8 * kPiece * (pieces after it)):
  // one multiplication per thread by a precomputed power, then an XOR reduction.
  if (c) c = gf2_mul(c, g_crc_tables.piece_pow[G - 1 - lt]);
#pragma unroll
  for (int o = 1; o < 32; o <<= 1)
    if (o < G) c ^= __shfl_xor_sync(0xFFFFFFFFu, c, o);
  if (G > 32) {  // groups of whole warps: XOR the warps' values
    if ((t & 31) == 0) sm[t >> 5] = c;
    __syncthreads();
    if (lt == 0)
      for (int w = 1; w < G / 32; ++w) c ^= sm[(t >> 5) + w];
  }
  if (lt == 0 && s < nseg) {
    if (single_level) out[s] = finish(c, L);
    else partial[s * blocks_per_seg + b] = c;
  }
}

// Level 2: one CTA per segment combines its blocks' crc0 values (right-aligned like level 1).
__global__ void __launch_bounds__(kThreads) crc_level2(int64_t nbytes, int64_t seg, int64_t nseg,
                                                       int64_t blocks_per_seg, const uint32_t* __restrict__ partial,
                                                       uint32_t* __restrict__ out) {
  __shared__ uint32_t sm[kThreads];
  __shared__ uint32_t mult[16];
  __shared__ uint32_t step;
  const int64_t s = blockIdx.x;
  const int t = threadIdx.x;
  const int64_t L = (s == nseg - 1) ? nbytes - s * seg : seg;
  const int64_t nb = cdiv(L, kBlock);
  const int64_t q = cdiv(nb, kThreads);  // blocks per thread
  const int64_t shift = q * kThreads - nb;
  if (t == 0) step = x8pow(uint64_t(kBlock));
  __syncthreads();
  uint32_t h = 0;
  for (int64_t v = int64_t(t) * q; v < int64_t(t + 1) * q; ++v) {
    const int64_t bi = v - shift;
    if (bi < 0) continue;  // leading virtual zero blocks
    h = (h ? gf2_mul(h, step) : 0u) ^ partial[s * blocks_per_seg + bi];
  }
  h = combine_group(h, kThreads, uint64_t(q) * kBlock, sm, mult);
  if (t == 0) out[s] = finish(h, L);
}

}  // namespace
}  // namespace zn

using namespace zn;

extern "C" {

size_t zn_crc32_temp_bytes(int64_t nbytes, int64_t segment_bytes) {
  if (nbytes <= 0 || segment_bytes <= 0) return 0;
  const int64_t nseg = cdiv(nbytes, segment_bytes);
  const int64_t seg = min(segment_bytes, nbytes);
  if (seg <= kBlock) return 0;
  return size_t(nseg * cdiv(seg, kBlock)) * sizeof(uint32_t);
}

int zn_crc32(const void* data, int64_t nbytes, int64_t segment_bytes, uint32_t* out, void* temp,
             size_t temp_bytes, void* stream) {
  if (nbytes < 0 || segment_bytes <= 0) return set_error(ZN_ERR_INVALID, "zn_crc32: bad arguments");
  if (nbytes == 0) return ZN_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint8_t* d = static_cast<const uint8_t*>(data);
  const int64_t nseg = cdiv(nbytes, segment_bytes);
  const int64_t seg = min(segment_bytes, nbytes);  // longest segment
  if (seg <= kBlock) {
    int G = 1;
    while (int64_t(G) * kPiece < seg) G <<= 1;
    const int64_t groups = kThreads / G;
    const int64_t grid = cdiv(nseg, groups);
    if (grid > 0x7FFFFFFF) return set_error(ZN_ERR_INVALID, "zn_crc32: too many segments");
    TimedLaunch tl("crc", st);
    crc_level1<<<unsigned(grid), kThreads, 0, st>>>(d, nbytes, segment_bytes, nseg, G, 1, true, out, nullptr);
    count_launch();
    return check_launch("zn_crc32");
  }
  const int64_t bps = cdiv(seg, kBlock);
  if (temp_bytes < size_t(nseg * bps) * sizeof(uint32_t) || !temp)
    return set_error(ZN_ERR_SPACE, "zn_crc32: temp buffer too small");
  if (nseg * bps > 0x7FFFFFFF) return set_error(ZN_ERR_INVALID, "zn_crc32: too many blocks");
  uint32_t* partial = static_cast<uint32_t*>(temp);
  {
    TimedLaunch tl("crc", st);  // both levels
    crc_level1<<<unsigned(nseg * bps), kThreads, 0, st>>>(d, nbytes, segment_bytes, nseg, kThreads, bps, false, out,
                                                          partial);
    crc_level2<<<unsigned(nseg), kThreads, 0, st>>>(nbytes, segment_bytes, nseg, bps, partial, out);
  }
  count_launch(2);
  return check_launch("zn_crc32");
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// zn_crc32_noalloc: the same two kernels with their partial-CRC scratch in a static device array,
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
  const int64_t nseg = cdiv(nbytes, segment_bytes);
  const int64_t seg = min(segment_bytes, nbytes);  // longest segment
  const int64_t bps = seg > kBlock ? cdiv(seg, kBlock) : 0;
  if (nseg * bps > kNoAllocSlots)
    return set_error(ZN_ERR_INVALID,
                     "zn_crc32_noalloc: %lld bytes in segments of %lld need %lld scratch slots (one per 32 KiB block "
                     "of each segment); the static scratch holds %lld (2 MiB). Use zn_crc32 with a temp buffer",
                     (long long)nbytes, (long long)segment_bytes, (long long)(nseg * bps), (long long)kNoAllocSlots);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint8_t* d = static_cast<const uint8_t*>(data);
  if (bps == 0) {  // every segment fits one CTA: the scratch is neither touched nor looked up
    int G = 1;
    while (int64_t(G) * kPiece < seg) G <<= 1;
    const int64_t grid = cdiv(nseg, int64_t(kThreads / G));
    if (grid > 0x7FFFFFFF) return set_error(ZN_ERR_INVALID, "zn_crc32_noalloc: too many segments");
    TimedLaunch tl("crc", st);
    crc_level1<<<unsigned(grid), kThreads, 0, st>>>(d, nbytes, segment_bytes, nseg, G, 1, true, out, nullptr);
    count_launch();
    return check_launch("zn_crc32_noalloc");
  }
  uint32_t* partial = nullptr;
  if (int rc = noalloc_scratch(&partial)) return rc;
  {
    TimedLaunch tl("crc", st);
    crc_level1<<<unsigned(nseg * bps), kThreads, 0, st>>>(d, nbytes, segment_bytes, nseg, kThreads, bps, false, out,
                                                          partial);
    crc_level2<<<unsigned(nseg), kThreads, 0, st>>>(nbytes, segment_bytes, nseg, bps, partial, out);
  }
  count_launch(2);
  return check_launch("zn_crc32_noalloc");
}
