// Compression: the fused whole-tensor path (zn_compress) and the batched ANS seam
// (zn_ans_compress).
//
// zn_compress replaces src/cuzipnn/_codec.py:308-413 (split, nvCOMP ANS, host passthrough
// decision and table build, two copy passes, prefix upload) with four kernels and no host round
// trip:
//   1. hist_kernel: one CTA per chunk counts the byte histograms of all K planes of its elements
//      (shared-memory atomics into lane-private columns) and writes one histogram per plane.
//   2. encode_kernel: one CTA per chunk turns each plane's histogram into a ZNR2 frequency table,
//      skips the planes whose entropy lower bound already fails the passthrough budget (they would
//      be stored raw anyway), rANS-encodes the others into a scratch slot per unit, and writes the
//      skipped (raw) planes straight to the blob offsets they have when every chunk codes the same
//      planes.
//   3. scan_kernel: one CTA per tensor applies the passthrough rule of _codec.py:361-372, writes
//      the header, the stored_bytes and comp_idx tables and the destination of every unit, and
//      checks the encoder's guessed raw-plane offsets against the final layout.
//   4. pack_kernel: one CTA per chunk copies the coded payloads from scratch into the blob, writes
//      the raw planes the encoder did not place (re-reading those elements), and zero-pads every
//      unit to 8 bytes.
#include <climits>
#include <type_traits>
#include <math.h>
#include <string.h>

#include <vector>

#include "zn_common.cuh"

namespace zn {
namespace {

constexpr int kEncThreads = 128;  // 4 warps per chunk
constexpr int kEncSym = 256 / kEncThreads;  // symbols per thread in table building
constexpr int kEncChains = 1;  // rANS states per lane (sub-chunks per lane)
static_assert(kEncChains == 1, "the staging ring holds one state per lane");
constexpr int kCols = 16;  // lane-private histogram columns

// One compression job (a tensor, or the chunk list of the batched seam).  Jobs live in device
// memory; a kernel's CTA finds its job by global chunk index (find_job).
struct EncArgs {
  const uint8_t* x;         // tensor elements
  const int64_t* in_ptrs;   // seam: chunk addresses (K == 1), else null
  const int64_t* in_bytes;  // seam: chunk sizes
  int64_t n;                // element count
  int64_t C;                // elements per chunk
  int64_t nch;              // chunks (units per plane)
  int64_t units;            // K * nch
  int64_t chunk0;           // global index of the job's first chunk
  int t;                    // log2(sub-chunks)
  int allow_skip;           // seam: 0 (every chunk is coded)
  double threshold;         // passthrough threshold
  uint8_t* meta;            // per unit, meta_slot bytes
  int64_t meta_slot;
  uint16_t* streams;        // per unit: unit_words words; per sub-chunk: sub_words; per lane: lane_words
  int64_t unit_words;
  int64_t sub_words;
  int64_t lane_words;
  int32_t* comp_bytes;      // per unit: payload bytes, or -1 if not coded
  uint32_t* part_hist;      // [nch][kHistParts][K][256] partial histograms from hist_kernel
  int64_t* dst_rel;         // per unit: offset from data_off, with bit 62 set if coded
  int64_t* scalars;         // [0] = data_off, [1] = size
  uint8_t* out;             // blob buffer
  uint64_t* size_out;       // device u64 receiving the blob size
  int64_t sizes_off, idx_off;
  // Raw planes written in place by the encoder: the blob offset a raw unit (b, j) has when every
  // chunk codes exactly one plane and all earlier planes are raw (spec_data_off + b *
  // spec_plane_bytes + j * align8(C)); scan checks the guess (scalars[2]) and pack skips them.
  int64_t spec_data_off, spec_plane_bytes;
  int header_len;
  uint8_t header[24 + 8 * 64];
};

// Parts per chunk of the histogram kernel (CTAs per chunk, each writing a partial histogram that
// the encoder sums).  One: with lane-private columns the counting keeps up, and fewer partial
// histograms are written and read back.
constexpr int kHistParts = 1;
constexpr int kHistThreads = 256;

struct EncSmem {
  uint32_t f[256];
  uint32_t fbuf[96];        // 256 12-bit fields
  uint32_t red_u[8];
  float red_f[8];
  unsigned long long red_ull[8];
  int npl[8];
  int skip[8];
  int nwsum[8];             // stream words per plane
  uint32_t stage[32][kEncThreads];  // per lane: last 32 emitted words, word h of lane t at [h % 32][t]
};

// ---- block-wide helpers (kEncThreads = 128 threads = 4 warps) ----------------------------------

__device__ __forceinline__ uint32_t block_sum_u(uint32_t v, uint32_t* red) {
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  uint32_t s = 0;
  for (int w = 0; w < kEncThreads / 32; ++w) s += red[w];
  return s;
}

__device__ __forceinline__ float block_sum_f(float v, float* red) {
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float s = 0.f;
  for (int w = 0; w < kEncThreads / 32; ++w) s += red[w];
  return s;
}

__device__ __forceinline__ unsigned long long block_max_ull(unsigned long long v, unsigned long long* red) {
  for (int o = 16; o; o >>= 1) {
    unsigned long long u = __shfl_xor_sync(0xFFFFFFFFu, v, o);
    v = u > v ? u : v;
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  unsigned long long s = 0;
  for (int w = 0; w < kEncThreads / 32; ++w) s = red[w] > s ? red[w] : s;
  return s;
}

// Exclusive scan of one value per thread over the block.
__device__ __forceinline__ uint32_t block_excl_scan(uint32_t v, uint32_t* red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  uint32_t incl = v;
  for (int o = 1; o < 32; o <<= 1) {
    uint32_t u = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += u;
  }
  __syncthreads();
  if (lane == 31) red[w] = incl;
  __syncthreads();
  uint32_t base = 0;
  for (int q = 0; q < w; ++q) base += red[q];
  return base + incl - v;
}

// ---- symbol access -------------------------------------------------------------------------

template <int K>
__device__ __forceinline__ uint64_t load_elem(const uint8_t* p) {
  uint64_t u = 0;
#pragma unroll
  for (int b = 0; b < K; ++b) u |= uint64_t(p[b]) << (8 * b);
  return u;
}

template <int K, bool REORDER>
__device__ __forceinline__ uint64_t reorder_elem(uint64_t u) {
  if constexpr (REORDER) {
    constexpr int W = 8 * K;
    uint64_t exp = (u >> (W - 9)) & 0xFF, sign = u >> (W - 1), mant = u & ((uint64_t(1) << (W - 9)) - 1);
    return (exp << (W - 8)) | (sign << (W - 9)) | mant;
  }
  return u;
}

// The 16 symbols of plane b for elements e0 .. e0 + 15 of a chunk (nact of them valid).
// mode: 2 = 16-byte loads, 1 = 8-byte loads, 0 = bytes.
// Byte plane b (after the exponent reorder) of 16 elements given as 4 * K little-endian words.
// bf16 has a direct form: the exponent byte of element u is (u >> 7) & 0xFF and the sign /
// mantissa byte (u >> 8 & 0x80) | (u & 0x7F), two elements per word.
template <int K, bool REORDER>
__device__ __forceinline__ void plane_of_elements(const uint32_t* e, int b, uint32_t* sym) {
  if constexpr (K == 2 && REORDER) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t t0 = e[2 * i], t1 = e[2 * i + 1];
      if (b == 1) {
        t0 >>= 7;
        t1 >>= 7;
      } else {
        t0 = (t0 & 0x007F007Fu) | ((t0 >> 8) & 0x00800080u);
        t1 = (t1 & 0x007F007Fu) | ((t1 >> 8) & 0x00800080u);
      }
      sym[i] = __byte_perm(t0, t1, 0x6420);
    }
  } else {
    uint32_t w[4 * K];
#pragma unroll
    for (int i = 0; i < 4 * K; ++i) w[i] = e[i];
    reorder_words<K, REORDER, true>(w, 4 * K);
    uint32_t p[K][4];
    elements_to_planes<K>(w, p);
#pragma unroll
    for (int q = 0; q < K; ++q)
      if (q == b) {
#pragma unroll
        for (int i = 0; i < 4; ++i) sym[i] = p[q][i];
      }
  }
}

template <int K, bool REORDER>
__device__ __forceinline__ void plane_symbols(const uint8_t* xc, int64_t e0, int nact, int b, int mode, uint32_t* sym) {
  if (nact == 16 && mode) {
    uint32_t e[4 * K];
    load_words(xc + e0 * K, e, 4 * K, mode == 2);
    plane_of_elements<K, REORDER>(e, b, sym);
    return;
  }
  uint64_t lo = 0, hi = 0;  // two 64-bit accumulators keep the runtime-indexed bytes in registers
  for (int i = 0; i < nact; ++i) {
    const uint64_t u = reorder_elem<K, REORDER>(load_elem<K>(xc + (e0 + i) * K));
    const uint64_t byte = (u >> (8 * b)) & 0xFF;
    if (i < 8) lo |= byte << (8 * i);
    else hi |= byte << (8 * (i - 8));
  }
  sym[0] = uint32_t(lo);
  sym[1] = uint32_t(lo >> 32);
  sym[2] = uint32_t(hi);
  sym[3] = uint32_t(hi >> 32);
}

// Histogram all planes over the chunk's whole VB-byte vectors; returns the elements covered.
// Each thread keeps kHistDepth independent vector loads in flight before its atomics.
constexpr int kHistDepth = 4;

// Histogram layout for K <= 2: byte offset sym << 8 | plane << 7 | lane << 2 (lane = threadIdx % 32),
// 64 KiB.  Every lane counts into its own column, so a warp's 32 atomics hit 32 different banks, and
// one byte permute builds the offset from the symbol byte and the lane's column byte.  K >= 4 keeps
// the [plane][sym][kCols] layout of 32-bit counters.
constexpr int kHist32Bytes = 256 * 256;

template <int KB>
__device__ __forceinline__ void hist32_add(uint8_t* hist, uint32_t src, uint32_t colw) {
  // Result bytes: [colw.b0, src.b(KB), 0, 0].
  const uint32_t off = __byte_perm(src, colw, 0x5504u | (uint32_t(KB) << 4));
  atomicAdd(reinterpret_cast<uint32_t*>(hist + off), 1u);
}

template <int K, bool REORDER, int VB>
__device__ __forceinline__ void hist_count(uint32_t (&w)[VB / 4], uint32_t* hist, int col) {
  if constexpr (K <= 2) {
    uint8_t* h8 = reinterpret_cast<uint8_t*>(hist);
    const uint32_t c0 = uint32_t(col) << 2, c1 = c0 | 128u;  // column bytes of planes 0 and 1
#pragma unroll
    for (int q = 0; q < VB / 4; ++q) {
      if constexpr (K == 2 && REORDER) {
        // bf16, two elements per word: exponent bytes (u >> 7) & 0xFF at bytes 0 and 2 of t,
        // sign / mantissa bytes (u >> 8 & 0x80) | (u & 0x7F) at bytes 0 and 2 of v.
        const uint32_t t = w[q] >> 7;
        const uint32_t v = (w[q] & 0x007F007Fu) | ((w[q] >> 8) & 0x00800080u);
        hist32_add<0>(h8, v, c0);
        hist32_add<0>(h8, t, c1);
        hist32_add<2>(h8, v, c0);
        hist32_add<2>(h8, t, c1);
      } else if constexpr (K == 2) {
        hist32_add<0>(h8, w[q], c0);
        hist32_add<1>(h8, w[q], c1);
        hist32_add<2>(h8, w[q], c0);
        hist32_add<3>(h8, w[q], c1);
      } else {
        hist32_add<0>(h8, w[q], c0);
        hist32_add<1>(h8, w[q], c0);
        hist32_add<2>(h8, w[q], c0);
        hist32_add<3>(h8, w[q], c0);
      }
    }
  } else {
    reorder_words<K, REORDER, true>(w, VB / 4);
#pragma unroll
    for (int q = 0; q < VB; ++q) {
      const uint32_t byte = (w[q >> 2] >> (8 * (q & 3))) & 0xFF;
      atomicAdd(&hist[(((q % K) << 8) | byte) * kCols + col], 1u);
    }
  }
}

// Count the VB-byte vectors of xc[0, m * K): kHistDepth vectors per thread per batch, the next
// batch's loads issued before the current batch is counted.  Returns the elements covered.
template <int K, bool REORDER, int VB>
__device__ __forceinline__ int64_t hist_vectors(const uint8_t* xc, int64_t m, uint32_t* hist, int col) {
  const int64_t nvec = m * K / VB;
  const int64_t step = kHistDepth * int64_t(blockDim.x);
  uint32_t w[kHistDepth][VB / 4], nx[kHistDepth][VB / 4];
  int64_t v0 = threadIdx.x;
#pragma unroll
  for (int d = 0; d < kHistDepth; ++d) {
    const int64_t v = v0 + d * int64_t(blockDim.x);
    if (v < nvec) load_words(xc + v * VB, nx[d], VB / 4, VB == 16);
  }
  for (; v0 < nvec; v0 += step) {
#pragma unroll
    for (int d = 0; d < kHistDepth; ++d)
#pragma unroll
      for (int i = 0; i < VB / 4; ++i) w[d][i] = nx[d][i];
#pragma unroll
    for (int d = 0; d < kHistDepth; ++d) {
      const int64_t v = v0 + step + d * int64_t(blockDim.x);
      if (v < nvec) load_words(xc + v * VB, nx[d], VB / 4, VB == 16);
    }
#pragma unroll
    for (int d = 0; d < kHistDepth; ++d) {
      if (v0 + d * int64_t(blockDim.x) >= nvec) break;
      hist_count<K, REORDER, VB>(w[d], hist, col);
    }
  }
  return nvec * VB / K;
}

// Part `blockIdx.y` of chunk `blockIdx.x`: histograms of all K planes of its elements, written as
// one partial histogram per plane (no global atomics; the encoder sums the parts).  The first
// kernel of a call: a single-job call passes its job by value (`one`), and CTA (0, 0) stores it
// into the table at `table` for the kernels after this one.
template <int K, bool REORDER>
__global__ void __launch_bounds__(kHistThreads) hist_kernel(const EncArgs* __restrict__ jobs, int njobs,
                                                           const __grid_constant__ FirstJob<EncArgs> one,
                                                           EncArgs* table) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint32_t* hist = reinterpret_cast<uint32_t*>(smem_raw);  // K <= 2: kHist32Bytes layout; else [K][256][kCols]
  if (one.valid && blockIdx.x == 0 && blockIdx.y == 0) store_job(one.job, table);
  const EncArgs& a = one.valid ? one.job : jobs[find_job(jobs, njobs, blockIdx.x)];
  const int64_t j = blockIdx.x - a.chunk0;
  const int part = blockIdx.y, tid = threadIdx.x;
  const uint8_t* xc;
  int64_t m;
  if (a.in_ptrs) {
    xc = reinterpret_cast<const uint8_t*>(a.in_ptrs[j]);
    m = a.in_bytes[j];
  } else {
    xc = a.x + j * a.C * K;
    m = min(a.C, a.n - j * a.C);
  }
  m = max(int64_t(0), min(m, a.C));
  const int64_t per = cdiv(cdiv(m, kHistParts), 16) * 16;
  const int64_t e0 = min(m, part * per), e1 = min(m, e0 + per);
  const uint8_t* xs = xc + e0 * K;
  const int64_t ms = e1 - e0;
  constexpr int kWords = K <= 2 ? kHist32Bytes / 4 : K * 256 * kCols;
  for (int i = tid; i < kWords; i += kHistThreads) hist[i] = 0;
  __syncthreads();
  const uintptr_t xa = reinterpret_cast<uintptr_t>(xs);
  const int mode = (xa & 15) == 0 ? 2 : (xa & 7) == 0 ? 1 : 0;
  const int col = K <= 2 ? (tid & 31) : (tid & (kCols - 1));
  int64_t done = 0;
  if (mode == 2) done = hist_vectors<K, REORDER, 16>(xs, ms, hist, col);
  else if (mode == 1) done = hist_vectors<K, REORDER, 8>(xs, ms, hist, col);
  for (int64_t e = done + tid; e < ms; e += kHistThreads) {
    const uint64_t u = reorder_elem<K, REORDER>(load_elem<K>(xs + e * K));
#pragma unroll
    for (int b = 0; b < K; ++b) {
      const uint32_t byte = uint32_t((u >> (8 * b)) & 0xFF);
      if constexpr (K <= 2) atomicAdd(&hist[(byte << 6) | (b << 5) | col], 1u);
      else atomicAdd(&hist[((b << 8) | byte) * kCols + col], 1u);
    }
  }
  __syncthreads();
  uint32_t* outp = a.part_hist + (j * kHistParts + part) * K * 256;
  for (int i = tid; i < K * 256; i += kHistThreads) {  // i = plane * 256 + symbol
    uint32_t c = 0;
    if constexpr (K <= 2) {
      const uint32_t* h = hist + ((i & 255) << 6) + ((i >> 8) << 5);
#pragma unroll
      for (int q = 0; q < 32; ++q) c += h[(q + i) & 31];
    } else {
#pragma unroll
      for (int q = 0; q < kCols; ++q) c += hist[i * kCols + ((q + i) & (kCols - 1))];
    }
    outp[i] = c;
  }
}

// One encode step of one state for symbol byte I (last symbol first; the decoder runs forward).
// A state at or above f * 2^19 (it would leave [L, 2^31) after coding) emits its low 16 bits into
// its own stream, which grows down from the end of the state's slot; the word goes to the lane's
// 32-word staging ring in shared memory (one predicated store of x, whose low half is the word, no
// branch; the rings interleave by lane, so every lane of a warp stores to its own bank).  Then
// x' = x + bias + q * (M - f) with q = floor(x / f) = umulhi(x, magic) >> shift, exact because
// x < 2^31; the shift sits in the low 5 bits of e.z, which the wrapping funnel shift uses.
template <bool FULL, int I>
__device__ __forceinline__ void encode_step(uint32_t& x, uint32_t& wp, uint32_t* stage, const uint32_t* sym,
                                            const uint4* tab, bool act) {
  const uint4 e = tab[get_byte(sym, I)];  // {magic, bias, (M - f) << 5 | shift, f * 2^19 - 1}
  const bool emit = (FULL || act) && x > e.w;
  wp -= emit;
  if (emit) stage[(wp & 31) * kEncThreads] = x;
  x = emit ? x >> 16 : x;
  const uint32_t q = __funnelshift_r(__umulhi(x, e.x), 0u, e.z);
  const uint32_t xn = x + e.y + q * (e.z >> 5);
  x = (FULL || act) ? xn : x;
}

// The 16-byte stream block of words h .. h + 7 (h a multiple of 8) from a lane's staging ring.
__device__ __forceinline__ uint4 stage_block(const uint32_t* st, uint32_t h) {
  const uint32_t* s = st + (h & 31) * kEncThreads;
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) w[i] = __byte_perm(s[2 * i * kEncThreads], s[(2 * i + 1) * kEncThreads], 0x5410);
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// 16 steps of the lane's kEncChains states, interleaved so the independent chains overlap.
template <bool FULL>
__device__ __forceinline__ void encode_round(uint32_t* x, uint32_t* wp, uint32_t* const* stage,
                                             const uint32_t (*sym)[4], const uint4* tab, const int* nact) {
#define ZN_ESTEP(I)                                                                                   \
  _Pragma("unroll") for (int c = 0; c < kEncChains; ++c)                                              \
      encode_step<FULL, I>(x[c], wp[c], stage[c], sym[c], tab, (I) < nact[c]);
  ZN_ESTEP(15) ZN_ESTEP(14) ZN_ESTEP(13) ZN_ESTEP(12) ZN_ESTEP(11) ZN_ESTEP(10) ZN_ESTEP(9) ZN_ESTEP(8)
  ZN_ESTEP(7) ZN_ESTEP(6) ZN_ESTEP(5) ZN_ESTEP(4) ZN_ESTEP(3) ZN_ESTEP(2) ZN_ESTEP(1) ZN_ESTEP(0)
#undef ZN_ESTEP
}

// The lean loop's 16 steps.  The staging position is kept as the byte offset
// tid * 4 + (wp % 32) * kEncThreads * 4 into the rows of the staging ring, so an emission costs
// one masked subtract and one store; wp is recovered at the end (a round emits at most 16 < 32
// words).
__device__ __forceinline__ void encode_round_lean(uint32_t& x, uint32_t& wp, uint8_t* rows, int tid,
                                                  const uint32_t* sym, const uint4* tab) {
  constexpr uint32_t kRowBytes = kEncThreads * 4, kRingBytes = 32 * kRowBytes;
  const uint32_t wo0 = uint32_t(tid) * 4 + (wp & 31) * kRowBytes;
  uint32_t wo = wo0;
#define ZN_LSTEP(I)                                                                               \
  {                                                                                               \
    const uint4 e = tab[get_byte(sym, I)];                                                        \
    const bool emit = x > e.w;                                                                    \
    wo = emit ? ((wo - kRowBytes) & (kRingBytes - 1)) : wo;                                       \
    if (emit) *reinterpret_cast<uint32_t*>(rows + wo) = x;                                        \
    x = emit ? x >> 16 : x;                                                                       \
    const uint32_t q = __funnelshift_r(__umulhi(x, e.x), 0u, e.z);                                \
    x = x + e.y + q * (e.z >> 5);                                                                 \
  }
  ZN_LSTEP(15) ZN_LSTEP(14) ZN_LSTEP(13) ZN_LSTEP(12) ZN_LSTEP(11) ZN_LSTEP(10) ZN_LSTEP(9) ZN_LSTEP(8)
  ZN_LSTEP(7) ZN_LSTEP(6) ZN_LSTEP(5) ZN_LSTEP(4) ZN_LSTEP(3) ZN_LSTEP(2) ZN_LSTEP(1) ZN_LSTEP(0)
#undef ZN_LSTEP
  wp -= (wo0 / kRowBytes - wo / kRowBytes) & 31u;
}

// ---- the encoder ----------------------------------------------------------------------------

template <int K, bool REORDER>
__global__ void __launch_bounds__(kEncThreads, 7) encode_kernel(const EncArgs* __restrict__ jobs, int njobs) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint4* etab = reinterpret_cast<uint4*>(smem_raw);                         // [K][256]
  EncSmem& S = *reinterpret_cast<EncSmem*>(smem_raw + K * 256 * 16);
  const EncArgs& a = jobs[find_job(jobs, njobs, blockIdx.x)];
  const int64_t j = blockIdx.x - a.chunk0;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint8_t* xc;
  int64_t m;
  if (a.in_ptrs) {
    xc = reinterpret_cast<const uint8_t*>(a.in_ptrs[j]);
    m = a.in_bytes[j];
  } else {
    xc = a.x + j * a.C * K;
    m = min(a.C, a.n - j * a.C);
  }
  if (m <= 0 || m > a.C) {
    if (tid < K) a.comp_bytes[tid * a.nch + j] = -1;
    return;
  }
  const uintptr_t xa = reinterpret_cast<uintptr_t>(xc);
  const int mode = (xa & 15) == 0 ? 2 : (xa & 7) == 0 ? 1 : 0;

  const Geom g = geom_of(m, a.t);
  const int64_t thr = a.allow_skip ? int64_t(double(m) * a.threshold) : INT64_MAX;

  // Phase B: per plane, frequencies, skip decision, coder table and payload header.  Thread t owns
  // symbols kEncSym * t .. kEncSym * t + kEncSym - 1.
  for (int b = 0; b < K; ++b) {
    const uint64_t u = uint64_t(b) * a.nch + j;
    uint8_t* meta = a.meta + u * a.meta_slot;
    uint32_t cc[kEncSym], ff[kEncSym];
    // Phase A: the plane's histogram is the sum of the parts' (hist_kernel).
    uint32_t npres = 0;
#pragma unroll
    for (int h = 0; h < kEncSym; ++h) {
      const int s = kEncSym * tid + h;
      uint32_t c = 0;
#pragma unroll
      for (int q = 0; q < kHistParts; ++q) c += a.part_hist[((j * kHistParts + q) * K + b) * 256 + s];
      cc[h] = c;
      npres += c > 0;
    }
    const uint32_t np = block_sum_u(npres, S.red_u);
    unsigned long long key = 0;
#pragma unroll
    for (int h = 0; h < kEncSym; ++h)
      if (cc[h]) {
        unsigned long long k2 = (static_cast<unsigned long long>(cc[h]) << 32) | uint32_t(255 - (kEncSym * tid + h));
        key = k2 > key ? k2 : key;
      }
    const int smax = 255 - int(block_max_ull(key, S.red_ull) & 0xFFFFFFFFu);
    // orc_normalize (oracle/zn_oracle.c) on the GPU.
#pragma unroll
    for (int h = 0; h < kEncSym; ++h) {
      const uint64_t q = (uint64_t(cc[h]) * kM + uint64_t(m / 2)) / uint64_t(m);
      ff[h] = cc[h] ? (q < 1 ? 1u : uint32_t(q)) : 0u;
    }
    if (np == 1) {
#pragma unroll
      for (int h = 0; h < kEncSym; ++h) ff[h] = (kEncSym * tid + h == smax) ? kM : 0u;
    } else {
      uint32_t fs = 0;
#pragma unroll
      for (int h = 0; h < kEncSym; ++h) fs += ff[h];
      const int64_t d = int64_t(kM) - int64_t(block_sum_u(fs, S.red_u));
      __syncthreads();
#pragma unroll
      for (int h = 0; h < kEncSym; ++h)
        if (kEncSym * tid + h == smax) S.f[0] = ff[h];
      __syncthreads();
      const int64_t fmax = S.f[0];
      if (fmax + d >= 1) {
#pragma unroll
        for (int h = 0; h < kEncSym; ++h)
          if (kEncSym * tid + h == smax) ff[h] = uint32_t(fmax + d);
      } else {
        fs = 0;
#pragma unroll
        for (int h = 0; h < kEncSym; ++h) {
          ff[h] = cc[h] ? 1u + uint32_t((uint64_t(cc[h]) * uint64_t(kM - np)) / uint64_t(m)) : 0u;
          fs += ff[h];
        }
        const int64_t sum2 = block_sum_u(fs, S.red_u);
#pragma unroll
        for (int h = 0; h < kEncSym; ++h)
          if (kEncSym * tid + h == smax) ff[h] += uint32_t(int64_t(kM) - sum2);
      }
    }
    // Cumulative frequencies and ranks of present symbols.
    uint32_t fsum = 0, psum = 0;
#pragma unroll
    for (int h = 0; h < kEncSym; ++h) {
      fsum += ff[h];
      psum += ff[h] > 0;
    }
    uint32_t cum = block_excl_scan(fsum, S.red_u);
    uint32_t rank = block_excl_scan(psum, S.red_u);
    // A lower bound of the payload size; planes that cannot beat the passthrough budget are not
    // coded (the blob is the same: such a unit is stored raw).  Per state, with y = log2(x) plus
    // 16 per emitted word: y starts at log2(L) = 15 and ends below 32 + 16 W (W words), and a
    // symbol of frequency f adds at least 12 - log2(f) - d bits, where the rounding of x / f costs
    // d <= -log2(1 - f / 2^15) without an emission (x >= 2^15) and, with one, the truncation and
    // the rounding (x >= 8 f) cost at most 2 * -log2(7 / 8) = 0.386 bits.  With I the sum of
    // 12 - log2(f) - d over the plane's symbols and S states: 16 W + 32 > (I + 15.772) / 1.024125
    // per state, so payload > meta + ((I + 15.772 S) / 1.024125 - 32 S) / 8 bytes.  64 bytes
    // cover the float rounding of the sums.
    float bits = 0.f;
#pragma unroll
    for (int h = 0; h < kEncSym; ++h)
      if (cc[h]) {
        const float fr = float(ff[h]);
        bits += float(cc[h]) * (float(kScaleBits) - log2f(fr) + log2f(1.f - fr * (1.f / 32768.f)));
      }
    const float info = block_sum_f(bits, S.red_f);
    const int64_t mb = meta_bytes(int(np), g);
    const float states = float(g.nu) * kLanes;
    const float lb = ((info + 15.772f * states) / 1.024125f - 32.f * states) * 0.125f + float(mb) - 64.f;
    const bool skip = lb >= float(thr);
    if (tid == 0) {
      S.skip[b] = skip;
      S.npl[b] = int(np);
    }
    if (skip) {
      if (tid == 0) a.comp_bytes[u] = -1;
      __syncthreads();
      continue;
    }
    // Encoder table: x' = x + bias + q * (M - f), q = floor(x / f) = umulhi(x, magic) >> shift
    // (division by multiplication: Granlund and Montgomery, "Division by invariant integers using
    // multiplication", 1994).  With shift = floor(log2 f) and magic = ceil(2^(32 + shift) / f) <
    // 2^32 (f not a power of two) the quotient is exact for x < 2^31, since x times the magic's
    // excess (< f <= 2^(shift + 1)) stays below 2^(32 + shift).  Powers of two use magic 2^31 and
    // shift log2(f) - 1; f = 1 uses magic 2^32 - 1 (q = x - 1) with the bias raised by M - 1.
    for (int i = tid; i < 96; i += kEncThreads) S.fbuf[i] = 0;
    __syncthreads();
#pragma unroll
    for (int h = 0; h < kEncSym; ++h) {
      const int s = kEncSym * tid + h;
      const uint32_t f = ff[h];
      uint4 e = make_uint4(0, 0, 0, 0);
      if (f == 1) {
        e = make_uint4(0xFFFFFFFFu, cum + kM - 1, (kM - 1) << 5, (1u << 19) - 1u);
      } else if (f > 1) {
        const uint32_t sh = 31 - __clz(f);  // floor(log2 f)
        const bool pow2 = (f & (f - 1)) == 0;
        const uint32_t mg = pow2 ? 0x80000000u : uint32_t(((uint64_t(1) << (32 + sh)) + f - 1) / f);
        e = make_uint4(mg, cum, ((kM - f) << 5) | (pow2 ? sh - 1 : sh), (f << 19) - 1u);
      }
      etab[b * 256 + s] = e;
      cum += f;
      // Payload header field: f - 1 as 12 bits at field index rank.
      if (f) {
        const uint32_t pos = 12 * rank++, v = f - 1;
        atomicOr(&S.fbuf[pos >> 5], v << (pos & 31));
        if ((pos & 31) > 20) atomicOr(&S.fbuf[(pos >> 5) + 1], v >> (32 - (pos & 31)));
      }
    }
    // Presence bitmap: symbol s = kEncSym * t + h is bit s; warp w covers symbols
    // 32 kEncSym w .. 32 kEncSym (w + 1) - 1, and its ballot h holds bit kEncSym * lane + h of them.
    uint32_t bm[kEncSym];
#pragma unroll
    for (int h = 0; h < kEncSym; ++h) bm[h] = __ballot_sync(0xFFFFFFFFu, ff[h] > 0);
    __syncthreads();
    if (lane < 4 * kEncSym) {  // this warp's bitmap byte `lane`: its symbols 8 lane .. 8 lane + 7
      uint32_t byte = 0;
#pragma unroll
      for (int bit = 0; bit < 8; ++bit) {
        const int k = 8 * lane + bit;
        byte |= ((bm[k % kEncSym] >> (k / kEncSym)) & 1u) << bit;
      }
      meta[2 + 4 * kEncSym * warp + lane] = uint8_t(byte);
    }
    const int64_t tb = table_bytes(int(np));
    for (int64_t i = tid; i < tb - 34; i += kEncThreads)
      meta[34 + i] = i < 384 ? uint8_t(S.fbuf[i >> 2] >> (8 * (i & 3))) : 0;
    if (tid == 0) {
      meta[0] = uint8_t(a.t);
      meta[1] = 0;
    }
    __syncthreads();
  }
  __syncthreads();

  // Phase C: encode.  A warp item is (plane, group of 8 sub-chunks); lane l of 8-lane segment g
  // runs chain c on sub-chunk 8 * group + 4 * c + g, each chain one state with its own stream slot.
  const int ngroups = int(cdiv(g.nu, 4 * kEncChains));
  int nplanes = 0, first_coded = K;
  uint32_t spec_mask = 0;  // skipped planes this CTA writes into the blob at their guessed offset
  for (int b = 0; b < K; ++b) {
    nplanes += !S.skip[b];
    if (!S.skip[b] && first_coded == K) first_coded = b;
  }
  if (a.allow_skip && a.out && nplanes > 0)
    for (int b = 0; b < K; ++b)
      if (S.skip[b]) spec_mask |= 1u << b;
  if (tid < K) {
    S.nwsum[tid] = 0;
    if ((spec_mask >> tid) & 1) a.comp_bytes[uint64_t(tid) * a.nch + j] = -2;
  }
  __syncthreads();
  const int seg = lane >> 3, l = lane & 7;
  const int rounds = int(g.sc / kRound);
  for (int item = warp; item < nplanes * ngroups; item += kEncThreads / 32) {
    int b = 0, seen = 0;
    for (int q = 0; q < K; ++q)
      if (!S.skip[q]) {
        if (seen == item / ngroups) b = q;
        ++seen;
      }
    const uint64_t u = uint64_t(b) * a.nch + j;
    const uint4* tab = etab + b * 256;
    int gi[kEncChains];
    bool valid[kEncChains];
    int64_t base[kEncChains], len[kEncChains];
    uint16_t* out[kEncChains];
    uint32_t* stage[kEncChains];
    uint32_t x[kEncChains], wp[kEncChains], flushed[kEncChains];
    uint32_t nxt[kEncChains][4 * K];
    uint8_t* spec0[kEncChains];  // this lane's bytes of plane 0 at the guessed blob place
    const bool spec_item = b == first_coded && spec_mask;
#pragma unroll
    for (int c = 0; c < kEncChains; ++c) {
      gi[c] = 4 * kEncChains * (item % ngroups) + 4 * c + seg;
      valid[c] = gi[c] < g.nu;
      base[c] = int64_t(gi[c]) * g.sc;
      len[c] = valid[c] ? min(g.sc, m - base[c]) : 0;
      out[c] = a.streams + u * a.unit_words + int64_t(gi[c]) * a.sub_words + int64_t(l) * a.lane_words;
      x[c] = kL;
      wp[c] = flushed[c] = uint32_t(a.lane_words);  // the stream grows down from the slot's end
      stage[c] = &S.stage[0][tid];  // one ring per lane: kEncChains == 1
      spec0[c] = spec_item ? a.out + a.spec_data_off + j * align8(a.C) + base[c] + l * kSteps : nullptr;
    }
    // The elements of the next (lower) round are loaded while the current round is encoded.
    auto full_round = [&](int c, int r) {
      return mode != 0 && len[c] - (int64_t(r) * kRound + l * kSteps) >= kSteps;
    };
#pragma unroll
    for (int c = 0; c < kEncChains; ++c)
      if (rounds > 0 && full_round(c, rounds - 1))
        load_words(xc + (base[c] + int64_t(rounds - 1) * kRound + l * kSteps) * K, nxt[c], 4 * K, mode == 2);
    // Rounds from the top; the partial rounds at the end of a sub-chunk come first, then the full
    // rounds run the lean loop below (no predication, running pointers).
    const int rfull = (kEncChains == 1 && mode != 0 && len[0] >= l * kSteps + kSteps)
                          ? int((len[0] - l * kSteps - kSteps) / kRound) + 1 : 0;
    int r = rounds - 1;
    for (; r >= rfull; --r) {
      uint32_t sym[kEncChains][4];
      int nact[kEncChains];
#pragma unroll
      for (int c = 0; c < kEncChains; ++c) {
        const int64_t off = int64_t(r) * kRound + l * kSteps;
        nact[c] = int(max(int64_t(0), min(int64_t(kSteps), len[c] - off)));
        if (full_round(c, r)) {
          plane_of_elements<K, REORDER>(nxt[c], b, sym[c]);
        } else {
          plane_symbols<K, REORDER>(xc, base[c] + off, nact[c], b, 0, sym[c]);
        }
        // The skipped (raw) planes of the same elements go to their guessed place in the blob.
        if (spec_item) {
#pragma unroll
          for (int q = 0; q < K; ++q) {
            if (!((spec_mask >> q) & 1)) continue;
            uint8_t* d = spec0[c] + q * a.spec_plane_bytes + int64_t(r) * kRound;
            uint32_t raw[4];
            if (full_round(c, r)) {
              plane_of_elements<K, REORDER>(nxt[c], q, raw);
              reinterpret_cast<uint2*>(d)[0] = make_uint2(raw[0], raw[1]);
              reinterpret_cast<uint2*>(d)[1] = make_uint2(raw[2], raw[3]);
            } else {
              plane_symbols<K, REORDER>(xc, base[c] + off, nact[c], q, 0, raw);
              for (int i = 0; i < nact[c]; ++i) d[i] = uint8_t(raw[i >> 2] >> (8 * (i & 3)));
            }
          }
        }
        if (r > 0 && full_round(c, r - 1))
          load_words(xc + (base[c] + int64_t(r - 1) * kRound + l * kSteps) * K, nxt[c], 4 * K, mode == 2);
      }
      if (nact[0] == kSteps && nact[kEncChains - 1] == kSteps) encode_round<true>(x, wp, stage, sym, tab, nact);
      else encode_round<false>(x, wp, stage, sym, tab, nact);
      // Completed 16-byte blocks of the staging ring go to the stream slot.
#pragma unroll
      for (int c = 0; c < kEncChains; ++c)
        while (flushed[c] - wp[c] >= 8) {
          flushed[c] -= 8;
          *reinterpret_cast<uint4*>(out[c] + flushed[c]) = stage_block(stage[c], flushed[c]);
        }
    }
    if constexpr (kEncChains == 1) {
      const uint8_t* xp = xc + (base[0] + int64_t(r) * kRound + l * kSteps) * K;  // round r's elements
      uint8_t* sp = spec_item ? spec0[0] + int64_t(r) * kRound : nullptr;
      // LAST: the coded plane is plane K - 1 and every other plane goes to the blob in place, from
      // 16-byte aligned elements (every float type's usual case): planes and loads fixed at compile
      // time.
      auto lean_rounds = [&](auto last) {
        constexpr bool LAST = decltype(last)::value;
        for (; r >= 0; --r) {
          uint32_t sym[1][4];
          plane_of_elements<K, REORDER>(nxt[0], LAST ? K - 1 : b, sym[0]);
          if (LAST || spec_item) {
#pragma unroll
            for (int q = 0; q < K; ++q) {
              if (LAST ? q == K - 1 : !((spec_mask >> q) & 1)) continue;
              uint32_t raw[4];
              plane_of_elements<K, REORDER>(nxt[0], q, raw);
              uint2* d = reinterpret_cast<uint2*>(sp + q * a.spec_plane_bytes);
              d[0] = make_uint2(raw[0], raw[1]);
              d[1] = make_uint2(raw[2], raw[3]);
            }
          }
          if (r > 0) load_words(xp - kRound * K, nxt[0], 4 * K, LAST || mode == 2);
          encode_round_lean(x[0], wp[0], reinterpret_cast<uint8_t*>(&S.stage[0][0]), tid, sym[0], tab);
          while (flushed[0] - wp[0] >= 8) {
            flushed[0] -= 8;
            *reinterpret_cast<uint4*>(out[0] + flushed[0]) = stage_block(stage[0], flushed[0]);
          }
          xp -= kRound * K;
          if (LAST || spec_item) sp -= kRound;
        }
      };
      if (b == K - 1 && spec_mask == (1u << (K - 1)) - 1 && mode == 2 && (K == 1 || spec_item))
        lean_rounds(std::true_type{});
      else
        lean_rounds(std::false_type{});
    }
#pragma unroll
    for (int c = 0; c < kEncChains; ++c)
      for (uint32_t h = wp[c]; h < flushed[c]; ++h) out[c][h] = uint16_t(stage[c][(h & 31) * kEncThreads]);
#pragma unroll
    for (int c = 0; c < kEncChains; ++c) {
      if (!valid[c]) continue;
      uint8_t* meta = a.meta + u * a.meta_slot;
      const uint32_t nwords = uint32_t(a.lane_words) - wp[c];
      const int64_t tb = table_bytes(S.npl[b]);
      const int64_t fi = int64_t(gi[c]) * kLanes + l;
      *reinterpret_cast<uint32_t*>(meta + tb + lengths_bytes(g) + 4 * fi) = x[c];
      if (g.lw == 2) *reinterpret_cast<uint16_t*>(meta + tb + 2 * fi) = uint16_t(nwords);
      else *reinterpret_cast<uint32_t*>(meta + tb + 4 * fi) = nwords;
      atomicAdd(&S.nwsum[b], int(nwords));
    }
  }
  __syncthreads();
  // Zero the pad of the length field area and publish the payload sizes.
  if (tid < K && !S.skip[tid]) {
    const int b = tid;
    const uint64_t u = uint64_t(b) * a.nch + j;
    uint8_t* meta = a.meta + u * a.meta_slot;
    const int npres = S.npl[b];
    const int64_t tb = table_bytes(npres);
    for (int64_t i = int64_t(g.nu) * kLanes * g.lw; i < lengths_bytes(g); ++i) meta[tb + i] = 0;
    a.comp_bytes[u] = int32_t(meta_bytes(npres, g) + 2 * int64_t(S.nwsum[b]));
  }
}

// ---- scan: passthrough rule, tables, destinations (src/cuzipnn/_codec.py:361-403) ------------

constexpr int kScanThreads = 1024;
constexpr int kScanPer = 4;

__device__ __forceinline__ void block_scan2(int64_t& a, int64_t& b, int64_t& ta, int64_t& tb, int64_t* sm) {
  // Exclusive scan of (a, b) over kScanThreads threads; totals returned in ta, tb.
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int64_t ia = a, ib = b;
  for (int o = 1; o < 32; o <<= 1) {
    int64_t ua = __shfl_up_sync(0xFFFFFFFFu, ia, o), ub = __shfl_up_sync(0xFFFFFFFFu, ib, o);
    if (lane >= o) { ia += ua; ib += ub; }
  }
  if (lane == 31) { sm[w] = ia; sm[32 + w] = ib; }
  __syncthreads();
  if (w == 0) {
    int64_t va = sm[lane], vb = sm[32 + lane];
    for (int o = 1; o < 32; o <<= 1) {
      int64_t ua = __shfl_up_sync(0xFFFFFFFFu, va, o), ub = __shfl_up_sync(0xFFFFFFFFu, vb, o);
      if (lane >= o) { va += ua; vb += ub; }
    }
    sm[64 + lane] = va;
    sm[96 + lane] = vb;
  }
  __syncthreads();
  const int64_t pa = w ? sm[64 + w - 1] : 0, pb = w ? sm[96 + w - 1] : 0;
  ta = sm[64 + 31];
  tb = sm[96 + 31];
  a = pa + ia - a;
  b = pb + ib - b;
  __syncthreads();
}

// One CTA per job.
__global__ void __launch_bounds__(kScanThreads) scan_kernel(const EncArgs* __restrict__ jobs) {
  __shared__ int64_t sm[128];
  __shared__ long long spec_lo, spec_hi;  // range of (guessed - final relative) offsets
  const EncArgs& a = jobs[blockIdx.x];
  const int tid = threadIdx.x;
  const int64_t last = a.n - (a.nch - 1) * a.C;
  int64_t carry_data = 0, carry_comp = 0;
  long long dlo = LLONG_MAX, dhi = LLONG_MIN;
  if (tid == 0) {
    spec_lo = LLONG_MAX;
    spec_hi = LLONG_MIN;
  }
  __syncthreads();
  for (int64_t start = 0; start < a.units; start += int64_t(kScanThreads) * kScanPer) {
    int64_t stored[kScanPer];
    bool use[kScanPer];
    int64_t sd = 0, sc = 0;
#pragma unroll
    for (int q = 0; q < kScanPer; ++q) {
      const int64_t i = start + int64_t(tid) * kScanPer + q;
      use[q] = false;
      stored[q] = 0;
      if (i < a.units) {
        const int64_t jj = i % a.nch;
        const int64_t raw = jj == a.nch - 1 ? last : a.C;
        const int64_t thr = __double2ll_rz(double(raw) * a.threshold);
        const int64_t c = a.comp_bytes[i];
        use[q] = c >= 0 && c < thr;
        stored[q] = use[q] ? c : raw;
        *reinterpret_cast<int32_t*>(a.out + a.sizes_off + 4 * i) = int32_t(stored[q]);
        sd += align8(stored[q]);
        sc += use[q];
      }
    }
    int64_t td, tc;
    block_scan2(sd, sc, td, tc, sm);
#pragma unroll
    for (int q = 0; q < kScanPer; ++q) {
      const int64_t i = start + int64_t(tid) * kScanPer + q;
      if (i < a.units) {
        a.dst_rel[i] = (carry_data + sd) | (int64_t(use[q]) << 62);
        if (a.comp_bytes[i] == -2) {  // written in place by the encoder: its guessed offset
          const int64_t gb = a.spec_data_off + (i / a.nch) * a.spec_plane_bytes + (i % a.nch) * align8(a.C);
          const long long d = gb - (carry_data + sd);
          dlo = d < dlo ? d : dlo;
          dhi = d > dhi ? d : dhi;
        }
        if (use[q]) *reinterpret_cast<int32_t*>(a.out + a.idx_off + 4 * (carry_comp + sc)) = int32_t(i);
        sd += align8(stored[q]);
        sc += use[q];
      }
    }
    carry_data += td;
    carry_comp += tc;
  }
  const int64_t n_comp = carry_comp;
  const int64_t data_off = align8(a.idx_off + 4 * n_comp);
  const int64_t size = data_off + carry_data;
  // The in-place raw units are usable only if every one of them landed where the blob has it.
  atomicMin(&spec_lo, dlo);
  atomicMax(&spec_hi, dhi);
  __syncthreads();
  for (int i = tid; i < a.header_len; i += kScanThreads) {
    uint8_t v = a.header[i];
    if (i >= 12 && i < 16) v = uint8_t(uint64_t(n_comp) >> (8 * (i - 12)));
    a.out[i] = v;
  }
  for (int64_t i = a.idx_off + 4 * n_comp + tid; i < data_off; i += kScanThreads) a.out[i] = 0;
  if (tid == 0) {
    a.scalars[0] = data_off;
    a.scalars[1] = size;
    a.scalars[2] = spec_lo == LLONG_MAX || (spec_lo == data_off && spec_hi == data_off);
    *a.size_out = uint64_t(size);
  }
}

// ---- pack (src/cuzipnn/_codec.py:381-403) ---------------------------------------------------

constexpr int kPackThreads = 256;

// Present symbols of a payload: the popcount of its bitmap, bytes [2, 34) of the 16-byte aligned
// meta block, read as three 16-byte loads.
__device__ __forceinline__ int count_present(const uint8_t* meta) {
  const uint4* m4 = reinterpret_cast<const uint4*>(meta);
  const uint4 a = m4[0], b = m4[1], c = m4[2];
  return __popc(a.x >> 16) + __popc(a.y) + __popc(a.z) + __popc(a.w) + __popc(b.x) + __popc(b.y) + __popc(b.z) +
         __popc(b.w) + __popc(c.x & 0xFFFFu);
}

// Warp-cooperative copy of L bytes (L even) from src to dst, both 2-byte aligned.  Each 16-byte
// aligned block of dst is assembled from the two aligned 16-byte source blocks it straddles (a
// funnel shift by their relative offset), so the body moves with 16-byte loads and stores; the
// ragged head and tail (under 16 bytes each) move by halfwords.  The source loads stay inside the
// 16-byte aligned span that holds the source bytes.
__device__ __forceinline__ uint4 shift_blocks(const uint4& A, const uint4& B, uint32_t q, uint32_t sh) {
  const uint32_t w0 = A.x, w1 = A.y, w2 = A.z, w3 = A.w, w4 = B.x, w5 = B.y, w6 = B.z, w7 = B.w;
  switch (q) {
    case 0: return make_uint4(__funnelshift_r(w0, w1, sh), __funnelshift_r(w1, w2, sh), __funnelshift_r(w2, w3, sh),
                              __funnelshift_r(w3, w4, sh));
    case 1: return make_uint4(__funnelshift_r(w1, w2, sh), __funnelshift_r(w2, w3, sh), __funnelshift_r(w3, w4, sh),
                              __funnelshift_r(w4, w5, sh));
    case 2: return make_uint4(__funnelshift_r(w2, w3, sh), __funnelshift_r(w3, w4, sh), __funnelshift_r(w4, w5, sh),
                              __funnelshift_r(w5, w6, sh));
    default: return make_uint4(__funnelshift_r(w3, w4, sh), __funnelshift_r(w4, w5, sh), __funnelshift_r(w5, w6, sh),
                               __funnelshift_r(w6, w7, sh));
  }
}

// Copy L bytes (even; dst and src 2-byte aligned) by G cooperating lanes (lane in [0, G), G >= 8 so
// that the head and the tail, at most 7 halfwords each, take one store per lane): halfword stores
// up to dst's 16-byte boundary, then 16-byte stores of the source shifted into place, then the
// tail.  Writes exactly [dst, dst + L).
template <int G = 32>
__device__ __forceinline__ void warp_copy16(uint8_t* __restrict__ dst, const uint8_t* __restrict__ src, int64_t L,
                                            int lane) {
  const int64_t h = min(L, int64_t((16 - (reinterpret_cast<uintptr_t>(dst) & 15)) & 15));
  if (2 * lane < h) reinterpret_cast<uint16_t*>(dst)[lane] = reinterpret_cast<const uint16_t*>(src)[lane];
  const int64_t nb = (L - h) >> 4;
  const uint8_t* s = src + h;
  const uint32_t r = uint32_t(reinterpret_cast<uintptr_t>(s) & 15);
  const uint4* sa = reinterpret_cast<const uint4*>(s - r);
  uint4* d = reinterpret_cast<uint4*>(dst + h);
  const uint32_t q = r >> 2, sh = (r & 3) * 8;
  for (int64_t k = lane; k < nb; k += G) {
    const uint4 A = sa[k];
    d[k] = r ? shift_blocks(A, sa[k + 1], q, sh) : A;
  }
  const int64_t t0 = h + nb * 16;
  if (2 * lane < L - t0)
    reinterpret_cast<uint16_t*>(dst + t0)[lane] = reinterpret_cast<const uint16_t*>(src + t0)[lane];
}

// Exclusive prefix sums of two values per thread (kPackThreads threads) into out[2 t], out[2 t + 1];
// out[2 * kPackThreads] gets the total.  Ends with a barrier.
__device__ void block_scan_pairs(int32_t v0, int32_t v1, int32_t* out, int32_t* warp_tot) {
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  int32_t incl = v0 + v1;
  for (int o = 1; o < 32; o <<= 1) {
    const int32_t x = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += x;
  }
  __syncthreads();
  if (lane == 31) warp_tot[w] = incl;
  __syncthreads();
  int32_t base = 0;
  for (int q = 0; q < w; ++q) base += warp_tot[q];
  const int32_t ex = base + incl - v0 - v1;
  out[2 * t] = ex;
  out[2 * t + 1] = ex + v0;
  if (t == kPackThreads - 1) out[2 * kPackThreads] = ex + v0 + v1;
  __syncthreads();
}

// Shared-memory staging of the payload copy: 16-byte blocks, filled by cp.async.
constexpr int kStageBlocks = 2048;  // 32 KiB

struct PayloadSmem {
  int32_t pre[2 * kPackThreads + 1];   // stream start, halfwords after the meta block
  int32_t bpre[2 * kPackThreads + 1];  // first staged block of each stream
  int32_t warp_tot[kPackThreads / 32];
  uint4 stage[kStageBlocks];
};

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t s = uint32_t(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}

// Copy one coded payload to dst (8-byte aligned): the meta block, then the nu * 8 streams, each
// from the tail of its scratch slot to its place after the meta block.  The 16-byte blocks that
// hold a window of streams are first fetched into shared memory with cp.async (all in flight at
// once, one wait), then each warp writes its streams out of shared memory, shifted into place.
// A stream longer than the window is copied straight from global memory.  Called by all
// kPackThreads threads of the CTA.
__device__ void copy_payload(const EncArgs& a, uint64_t u, int64_t m, uint8_t* dst, int npres, PayloadSmem& P) {
  const uint8_t* meta = a.meta + u * a.meta_slot;
  const Geom g = geom_of(m, a.t);
  const int64_t tb = table_bytes(npres);
  const int64_t mh = meta_bytes(npres, g) / 2;
  const int S = g.nu * kLanes, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nwarps = kPackThreads / 32;
  if (warp == nwarps - 1) warp_copy16(dst, meta, 2 * mh, lane);
  const uint16_t* streams = a.streams + u * a.unit_words;
  auto src_of = [&](int fi, int32_t n) {
    return reinterpret_cast<const uint8_t*>(streams + int64_t(fi / kLanes) * a.sub_words +
                                            int64_t(fi % kLanes) * a.lane_words + (a.lane_words - n));
  };
  auto len_of = [&](int fi) {
    return fi >= S ? 0 : g.lw == 2 ? int32_t(reinterpret_cast<const uint16_t*>(meta + tb)[fi])
                                   : int32_t(reinterpret_cast<const uint32_t*>(meta + tb)[fi]);
  };
  int32_t n2[2], nb2[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int fi = 2 * tid + h;
    n2[h] = len_of(fi);
    const uintptr_t s0 = n2[h] ? reinterpret_cast<uintptr_t>(src_of(fi, n2[h])) : 0;
    nb2[h] = n2[h] ? int32_t(((s0 + 2 * uint32_t(n2[h]) + 15) >> 4) - (s0 >> 4)) : 0;
  }
  block_scan_pairs(n2[0], n2[1], P.pre, P.warp_tot);
  block_scan_pairs(nb2[0], nb2[1], P.bpre, P.warp_tot);
  for (int fa = 0; fa < S;) {
    // The window: streams [fa, fb) whose blocks fit in the staging buffer (at least stream fa).
    int fb = fa + 1;
    for (int st = 256; st > 0; st >>= 1)
      if (fb + st <= S && P.bpre[fb + st] - P.bpre[fa] <= kStageBlocks) fb += st;
    const int32_t b0 = P.bpre[fa], nb = P.bpre[fb] - b0;
    if (nb > kStageBlocks) {  // one stream longer than the window: straight from global memory
      const int32_t n = P.pre[fa + 1] - P.pre[fa];
      if (warp == 0) warp_copy16(dst + 2 * (mh + int64_t(P.pre[fa])), src_of(fa, n), 2 * int64_t(n), lane);
    } else {
      // Groups of 8 threads, one stream each: stage the stream's 16-byte blocks, then copy it out.
      const int grp = tid >> 3, g8 = tid & 7;
      for (int fi = fa + grp; fi < fb; fi += kPackThreads / 8) {
        const int32_t n = P.pre[fi + 1] - P.pre[fi];
        if (!n) continue;
        const uint8_t* s0 = reinterpret_cast<const uint8_t*>(reinterpret_cast<uintptr_t>(src_of(fi, n)) & ~uintptr_t(15));
        const int32_t nbf = P.bpre[fi + 1] - P.bpre[fi];
        for (int32_t k = g8; k < nbf; k += 8) cp_async16(&P.stage[P.bpre[fi] - b0 + k], s0 + 16 * int64_t(k));
      }
      asm volatile("cp.async.commit_group;\n" ::: "memory");
      asm volatile("cp.async.wait_group 0;\n" ::: "memory");
      __syncthreads();
      for (int fi = fa + grp; fi < fb; fi += kPackThreads / 8) {
        const int32_t n = P.pre[fi + 1] - P.pre[fi];
        if (!n) continue;
        const uintptr_t off = reinterpret_cast<uintptr_t>(src_of(fi, n)) & 15;
        warp_copy16<8>(dst + 2 * (mh + int64_t(P.pre[fi])),
                       reinterpret_cast<const uint8_t*>(&P.stage[P.bpre[fi] - b0]) + off, 2 * int64_t(n), g8);
      }
    }
    __syncthreads();
    fa = fb;
  }
}

// kPackParts CTAs per chunk, the parts of a chunk adjacent in launch order: part p of chunk j
// splits out 1/kPackParts of the chunk's elements for the raw planes, and part 0 also copies the
// chunk's coded payloads.  Chunks run in reverse order, so the most recently encoded (and read)
// chunks are still in L2.  One part: when the encoder has placed the raw planes (the usual case)
// extra parts only add CTAs with nothing to do (7B bf16: 2.09 ms with 4 parts, 1.69 ms with 1).
constexpr int kPackParts = 1;
template <int K>
constexpr int kPackGroups = K >= 4 ? 1 : 4 / K;

template <int K, bool REORDER>
__global__ void __launch_bounds__(kPackThreads, 5) pack_kernel(const EncArgs* __restrict__ jobs, int njobs, int64_t total_chunks) {
  __shared__ PayloadSmem P;
  const int64_t gj = total_chunks - 1 - blockIdx.x / kPackParts;
  const EncArgs& a = jobs[find_job(jobs, njobs, gj)];
  const int64_t j = gj - a.chunk0;
  const int part = int(blockIdx.x % kPackParts);
  const int64_t m = min(a.C, a.n - j * a.C);
  const int64_t data_off = a.scalars[0];
  __shared__ int npres[K];
  uint8_t* dst[K];
  bool coded[K], raw_w[K];  // raw_w: a raw plane this kernel writes (not already in place)
  bool any_raw = false, any_coded = false;
  const bool spec_ok = a.scalars[2] != 0;
  if (part == 0 && threadIdx.x < K) {
    const uint64_t u = uint64_t(threadIdx.x) * a.nch + j;
    npres[threadIdx.x] = (a.dst_rel[u] >> 62) & 1 ? count_present(a.meta + u * a.meta_slot) : 0;
  }
#pragma unroll
  for (int b = 0; b < K; ++b) {
    const uint64_t u = uint64_t(b) * a.nch + j;
    const int64_t d = a.dst_rel[u];
    coded[b] = (d >> 62) & 1;
    dst[b] = a.out + data_off + (d & ((int64_t(1) << 62) - 1));
    raw_w[b] = !coded[b] && !(spec_ok && a.comp_bytes[u] == -2);
    any_raw |= raw_w[b];
    any_coded |= coded[b];
  }
  // Raw planes: this part's 16-element groups, kPackGroups per thread per pass (128 input bytes).
  // The first pass's loads are issued before the payload copy so that the two overlap.
  constexpr int G = kPackGroups<K>;
  const uint8_t* xc = a.x + j * a.C * K;
  const uintptr_t xa = reinterpret_cast<uintptr_t>(xc);
  const int mode = (xa & 15) == 0 ? 2 : (xa & 7) == 0 ? 1 : 0;
  const int64_t ngrp = (mode && any_raw) ? m / 16 : 0;
  const int64_t gper = cdiv(ngrp, kPackParts);
  const int64_t g0 = part * gper, g1 = min(ngrp, g0 + gper);
  uint32_t e[G][4 * K];
  int64_t vb = g0 + threadIdx.x;
#pragma unroll
  for (int d = 0; d < G; ++d) {
    const int64_t v = vb + d * kPackThreads;
    if (v < g1) load_words(xc + v * 16 * K, e[d], 4 * K, mode == 2);
  }
  // Coded payloads: part 0 copies them whole (one prefix computation per payload).
  if (any_coded && part == 0) {
    __syncthreads();  // npres
#pragma unroll
    for (int b = 0; b < K; ++b) {
      if (!coded[b]) continue;
      const uint64_t u = uint64_t(b) * a.nch + j;
      const int64_t size = a.comp_bytes[u];
      copy_payload(a, u, m, dst[b], npres[b], P);
      if (threadIdx.x < 8 && size + threadIdx.x < align8(size)) dst[b][size + threadIdx.x] = 0;
    }
  }
  for (; any_raw && vb < g1; vb += G * kPackThreads) {
    if (vb != g0 + threadIdx.x) {
#pragma unroll
      for (int d = 0; d < G; ++d) {
        const int64_t v = vb + d * kPackThreads;
        if (v < g1) load_words(xc + v * 16 * K, e[d], 4 * K, mode == 2);
      }
    }
#pragma unroll
    for (int d = 0; d < G; ++d) {
      const int64_t v = vb + d * kPackThreads;
      if (v >= g1) break;
      reorder_words<K, REORDER, true>(e[d], 4 * K);
      uint32_t p[K][4];
      elements_to_planes<K>(e[d], p);
#pragma unroll
      for (int b = 0; b < K; ++b)
        if (raw_w[b]) {
          uint8_t* q = dst[b] + v * 16;
          if ((reinterpret_cast<uintptr_t>(q) & 15) == 0) *reinterpret_cast<uint4*>(q) = make_uint4(p[b][0], p[b][1], p[b][2], p[b][3]);
          else {
            reinterpret_cast<uint2*>(q)[0] = make_uint2(p[b][0], p[b][1]);
            reinterpret_cast<uint2*>(q)[1] = make_uint2(p[b][2], p[b][3]);
          }
        }
    }
  }
  if (part != kPackParts - 1) return;
  for (int64_t e1 = (mode ? m / 16 : 0) * 16 + threadIdx.x; any_raw && e1 < m; e1 += kPackThreads) {
    const uint64_t w = reorder_elem<K, REORDER>(load_elem<K>(xc + e1 * K));
#pragma unroll
    for (int b = 0; b < K; ++b)
      if (raw_w[b]) dst[b][e1] = uint8_t(w >> (8 * b));
  }
  if (threadIdx.x < 8 && m + threadIdx.x < align8(m)) {
#pragma unroll
    for (int b = 0; b < K; ++b)
      if (!coded[b]) dst[b][m + threadIdx.x] = 0;
  }
}

// ---- batched seam: assemble each payload into the caller's out_ptrs[i] ---------------------

__global__ void __launch_bounds__(kPackThreads) assemble_kernel(const EncArgs* __restrict__ job, const int64_t* in_bytes,
                                                                const int64_t* out_ptrs, int64_t* out_bytes,
                                                                int32_t* statuses) {
  const EncArgs& a = *job;
  const int64_t i = blockIdx.x;
  const int64_t size = a.comp_bytes[i];
  if (size < 0) {
    if (threadIdx.x == 0) { out_bytes[i] = 0; statuses[i] = 1; }
    return;
  }
  __shared__ int npres;
  __shared__ PayloadSmem P;
  if (threadIdx.x == 0) npres = count_present(a.meta + uint64_t(i) * a.meta_slot);
  __syncthreads();
  copy_payload(a, uint64_t(i), in_bytes[i], reinterpret_cast<uint8_t*>(out_ptrs[i]), npres, P);
  if (threadIdx.x == 0) { out_bytes[i] = size; statuses[i] = 0; }
}

// ---- host-side launch helpers ---------------------------------------------------------------

struct EncLayout {
  int64_t meta_slot, unit_words, sub_words, lane_words;
  size_t off_comp, off_dst, off_scalars, off_hist, off_meta, off_streams, total;
};

// Scratch of one job with `units` (plane, chunk) units of chunk length C and 2^t sub-chunks.
EncLayout enc_layout(int64_t units, int64_t C, int t) {
  EncLayout L;
  // A shorter last unit can have more (smaller) sub-chunks than a full one, so the slots are
  // sized for 2^t sub-chunks of the full unit's sub-chunk length.
  const Geom g = geom_of(C, t);
  L.meta_slot = (max_meta_bytes(t) + 15) & ~int64_t(15);
  L.lane_words = ((g.sc / kLanes) + 7) & ~int64_t(7);  // multiple of 8 words: 16-byte aligned slots
  L.sub_words = kLanes * L.lane_words;
  L.unit_words = L.sub_words << t;
  size_t o = 0;
  auto take = [&](size_t bytes) { size_t r = o; o = (o + bytes + 255) & ~size_t(255); return r; };
  L.off_comp = take(size_t(units) * 4);
  L.off_dst = take(size_t(units) * 8);
  L.off_scalars = take(64);
  L.off_hist = take(size_t(units) * kHistParts * 256 * 4);
  L.off_meta = take(size_t(units) * size_t(L.meta_slot));
  L.off_streams = take(size_t(units) * size_t(L.unit_words) * 2);
  L.total = o;
  return L;
}

size_t enc_smem(int K) { return size_t(K) * 256 * 16 + sizeof(EncSmem); }
size_t hist_smem(int K) { return K <= 2 ? size_t(kHist32Bytes) : size_t(K) * 256 * kCols * 4; }


int sub_log2(int sub_chunks) {
  for (int t = kMinSubLog2; t <= kMaxSubLog2; ++t)
    if (sub_chunks == (1 << t)) return t;
  return -1;
}

// Point a job's scratch pointers at its region of the temp buffer.
void bind_scratch(EncArgs& a, uint8_t* region, int64_t units) {
  const EncLayout L = enc_layout(units, a.C, a.t);
  a.meta = region + L.off_meta;
  a.meta_slot = L.meta_slot;
  a.streams = reinterpret_cast<uint16_t*>(region + L.off_streams);
  a.unit_words = L.unit_words;
  a.sub_words = L.sub_words;
  a.lane_words = L.lane_words;
  a.comp_bytes = reinterpret_cast<int32_t*>(region + L.off_comp);
  a.part_hist = reinterpret_cast<uint32_t*>(region + L.off_hist);
  a.dst_rel = reinterpret_cast<int64_t*>(region + L.off_dst);
  a.scalars = reinterpret_cast<int64_t*>(region + L.off_scalars);
}

template <int K, bool REORDER>
int launch_encode(EncArgs* jobs, int njobs, int64_t grid, cudaStream_t s, const EncArgs* one = nullptr) {
  if (grid <= 0) return ZN_OK;
  const size_t hs = hist_smem(K);
  auto hf = hist_kernel<K, REORDER>;
  if (int rc = set_max_smem(reinterpret_cast<const void*>(hf), int(hs))) return rc;
  FirstJob<EncArgs> fj{};
  if (one) {
    fj.job = *one;
    fj.valid = 1;
  }
  {
    TimedLaunch tl("hist", s);
    hf<<<dim3(unsigned(grid), kHistParts), kHistThreads, hs, s>>>(jobs, njobs, fj, jobs);
  }
  const size_t sm = enc_smem(K);
  auto fn = encode_kernel<K, REORDER>;
  if (int rc = set_max_smem(reinterpret_cast<const void*>(fn), int(sm))) return rc;
  {
    TimedLaunch tl("encode", s);
    fn<<<unsigned(grid), kEncThreads, sm, s>>>(jobs, njobs);
  }
  count_launch(2);
  return check_launch("encode_kernel");
}

template <int K, bool REORDER>
void launch_pack(const EncArgs* jobs, int njobs, int64_t grid, cudaStream_t s) {
  if (grid <= 0) return;
  TimedLaunch tl("pack", s);
  pack_kernel<K, REORDER><<<unsigned(grid * kPackParts), kPackThreads, 0, s>>>(jobs, njobs, grid);
  count_launch();
}

bool valid_k(int k, int reorder) { return (k == 1 || k == 2 || k == 4 || k == 8) && !(reorder && k != 2 && k != 4); }

}  // namespace
}  // namespace zn

using namespace zn;

extern "C" {

int64_t zn_ans_max_compressed_chunk_bytes(int64_t chunk_bytes, int sub_chunks) {
  const int t = sub_log2(sub_chunks);
  if (t < 0 || chunk_bytes <= 0 || chunk_bytes > kMaxChunkBytes) return -1;
  return max_payload(chunk_bytes, t);
}

size_t zn_ans_compress_temp_bytes(int64_t count, int64_t chunk_bytes, int sub_chunks) {
  const int t = sub_log2(sub_chunks);
  if (t < 0 || count < 0 || chunk_bytes <= 0) return 0;
  return job_table_bytes<EncArgs>(1, count) + enc_layout(count, chunk_bytes, t).total;
}

int zn_ans_compress(const int64_t* in_ptrs, const int64_t* in_bytes, int64_t chunk_bytes, int64_t count,
                    const int64_t* out_ptrs, int64_t* out_bytes, int32_t* statuses, int sub_chunks, void* temp,
                    size_t temp_bytes, void* stream) {
  const int t = sub_log2(sub_chunks);
  if (t < 0 || count < 0 || count > 0x7FFFFFFF || chunk_bytes <= 0 || chunk_bytes > kMaxChunkBytes)
    return set_error(ZN_ERR_INVALID, "zn_ans_compress: bad arguments");
  if (count == 0) return ZN_OK;
  if (!temp || temp_bytes < zn_ans_compress_temp_bytes(count, chunk_bytes, sub_chunks))
    return set_error(ZN_ERR_SPACE, "zn_ans_compress: temp buffer too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* tb = static_cast<uint8_t*>(temp);
  EncArgs a{};
  a.in_ptrs = in_ptrs;
  a.in_bytes = in_bytes;
  a.C = chunk_bytes;
  a.nch = a.units = count;
  a.t = t;
  a.allow_skip = 0;
  a.threshold = 1.0;
  bind_scratch(a, tb + job_table_bytes<EncArgs>(1, count), count);
  EncArgs* dj = reinterpret_cast<EncArgs*>(tb);
  if (int rc = upload_jobs(&a, 1, dj, count, s)) return rc;
  if (int rc = launch_encode<1, false>(dj, 1, count, s)) return rc;
  assemble_kernel<<<unsigned(count), kPackThreads, 0, s>>>(dj, in_bytes, out_ptrs, out_bytes, statuses);
  count_launch();
  return check_launch("zn_ans_compress");
}

int64_t zn_compress_bound(int64_t n, int k, int ndim, int64_t chunk_bytes) {
  if (n < 0 || k <= 0 || ndim < 0 || chunk_bytes <= 0) return -1;
  const int64_t nch = cdiv(n, chunk_bytes), total = int64_t(k) * nch;
  const int64_t head = align8(24 + 8 * int64_t(ndim) + 8 * total);
  const int64_t data = nch ? int64_t(k) * ((nch - 1) * align8(chunk_bytes) + align8(n - (nch - 1) * chunk_bytes)) : 0;
  return head + data;
}

size_t zn_compress_batch_temp_bytes(int njobs, const int64_t* n, int k, int64_t chunk_bytes, int sub_chunks) {
  const int t = sub_log2(sub_chunks);
  if (t < 0 || njobs < 0 || k <= 0 || chunk_bytes <= 0) return 0;
  size_t total = 0;
  int64_t chunks = 0;
  for (int i = 0; i < njobs; ++i) {
    if (n[i] < 0) return 0;
    chunks += cdiv(n[i], chunk_bytes);
    total += enc_layout(int64_t(k) * cdiv(n[i], chunk_bytes), chunk_bytes, t).total;
  }
  return total + job_table_bytes<EncArgs>(njobs, chunks);
}

size_t zn_compress_temp_bytes(int64_t n, int k, int64_t chunk_bytes, int sub_chunks) {
  return zn_compress_batch_temp_bytes(1, &n, k, chunk_bytes, sub_chunks);
}

int zn_compress_batch(int njobs, const void* const* x, const int64_t* n, int k, int reorder, const void* const* headers,
                      const int* header_bytes, int64_t chunk_bytes, int sub_chunks, double threshold, void* const* out,
                      const int64_t* out_capacity, uint64_t* sizes_out, void* temp, size_t temp_bytes, void* stream) {
  const int t = sub_log2(sub_chunks);
  if (njobs < 0 || t < 0 || !valid_k(k, reorder) || chunk_bytes <= 0 || chunk_bytes > kMaxChunkBytes ||
      chunk_bytes % 8 || !(threshold > 0.0 && threshold <= 1.0))
    return set_error(ZN_ERR_INVALID, "zn_compress: bad arguments");
  if (njobs == 0) return ZN_OK;
  NvtxScope range("zn_compress_batch");
  if (!temp || temp_bytes < zn_compress_batch_temp_bytes(njobs, n, k, chunk_bytes, sub_chunks))
    return set_error(ZN_ERR_SPACE, "zn_compress: temp buffer too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* tb = static_cast<uint8_t*>(temp);
  int64_t total_chunks = 0;
  for (int i = 0; i < njobs; ++i) total_chunks += cdiv(n[i], chunk_bytes);
  uint8_t* region = tb + job_table_bytes<EncArgs>(njobs, total_chunks);
  std::vector<EncArgs> jobs(static_cast<size_t>(njobs));
  int64_t chunk0 = 0;
  for (int i = 0; i < njobs; ++i) {
    const int hb = header_bytes[i];
    if (n[i] < 0 || hb < 24 || hb > 24 + 8 * 64 || (hb - 24) % 8 || (reinterpret_cast<uintptr_t>(x[i]) & 7) ||
        (reinterpret_cast<uintptr_t>(out[i]) & 7))
      return set_error(ZN_ERR_INVALID, "zn_compress: bad arguments (job %d)", i);
    if (out_capacity[i] < zn_compress_bound(n[i], k, (hb - 24) / 8, chunk_bytes))
      return set_error(ZN_ERR_SPACE, "zn_compress: output buffer too small (job %d)", i);
    EncArgs& a = jobs[size_t(i)];
    memset(&a, 0, sizeof(a));
    a.x = static_cast<const uint8_t*>(x[i]);
    a.n = n[i];
    a.C = chunk_bytes;
    a.nch = cdiv(n[i], chunk_bytes);
    a.units = int64_t(k) * a.nch;
    a.chunk0 = chunk0;
    a.t = t;
    a.allow_skip = 1;
    a.threshold = threshold;
    bind_scratch(a, region, a.units);
    region += enc_layout(a.units, chunk_bytes, t).total;
    a.out = static_cast<uint8_t*>(out[i]);
    a.size_out = sizes_out + i;
    a.sizes_off = hb;
    a.idx_off = hb + 4 * a.units;
    a.spec_data_off = align8(a.idx_off + 4 * a.nch);
    a.spec_plane_bytes = a.nch ? (a.nch - 1) * align8(chunk_bytes) + align8(n[i] - (a.nch - 1) * chunk_bytes) : 0;
    a.header_len = hb;
    memcpy(a.header, headers[i], size_t(hb));
    chunk0 += a.nch;
  }
  if (chunk0 > 0x7FFFFFFF / kPackParts) return set_error(ZN_ERR_INVALID, "zn_compress: too many chunks");
  EncArgs* dj = reinterpret_cast<EncArgs*>(tb);
  // A single job with chunks goes to the histogram kernel by value (it stores the table itself).
  const EncArgs* one = njobs == 1 && chunk0 > 0 ? jobs.data() : nullptr;
  if (!one)
    if (int rc = upload_jobs(jobs.data(), njobs, dj, chunk0, s)) return rc;
  int rc = ZN_OK;
  switch (k * 2 + (reorder ? 1 : 0)) {
    case 2: rc = launch_encode<1, false>(dj, njobs, chunk0, s, one); break;
    case 4: rc = launch_encode<2, false>(dj, njobs, chunk0, s, one); break;
    case 5: rc = launch_encode<2, true>(dj, njobs, chunk0, s, one); break;
    case 8: rc = launch_encode<4, false>(dj, njobs, chunk0, s, one); break;
    case 9: rc = launch_encode<4, true>(dj, njobs, chunk0, s, one); break;
    default: rc = launch_encode<8, false>(dj, njobs, chunk0, s, one); break;
  }
  if (rc) return rc;
  {
    TimedLaunch tl("scan", s);
    scan_kernel<<<unsigned(njobs), kScanThreads, 0, s>>>(dj);
  }
  count_launch();
  if ((rc = check_launch("scan_kernel"))) return rc;
  switch (k * 2 + (reorder ? 1 : 0)) {
    case 2: launch_pack<1, false>(dj, njobs, chunk0, s); break;
    case 4: launch_pack<2, false>(dj, njobs, chunk0, s); break;
    case 5: launch_pack<2, true>(dj, njobs, chunk0, s); break;
    case 8: launch_pack<4, false>(dj, njobs, chunk0, s); break;
    case 9: launch_pack<4, true>(dj, njobs, chunk0, s); break;
    default: launch_pack<8, false>(dj, njobs, chunk0, s); break;
  }
  return check_launch("pack_kernel");
}

int zn_compress(const void* x, int64_t n, int k, int reorder, const void* header, int header_bytes,
                int64_t chunk_bytes, int sub_chunks, double threshold, void* out, int64_t out_capacity,
                uint64_t* size_out, void* temp, size_t temp_bytes, void* stream) {
  return zn_compress_batch(1, &x, &n, k, reorder, &header, &header_bytes, chunk_bytes, sub_chunks, threshold, &out,
                           &out_capacity, size_out, temp, temp_bytes, stream);
}

}  // extern "C"
