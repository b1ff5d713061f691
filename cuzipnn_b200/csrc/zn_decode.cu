// Decompression: the fused whole-tensor path (zn_decompress) and the batched ANS seam
// (zn_ans_decompress).
//
// zn_decompress replaces src/cuzipnn/_codec.py:471-530 (table upload, cumsum, nvCOMP ANS decode
// into a planar buffer, then the Triton merge) with two kernels:
//   1. dscan_kernel: one CTA turns the blob's stored_bytes and comp_idx tables into the blob
//      offset of every (plane, chunk) unit, flags the rANS-coded ones and validates the tables.
//   2. decode_kernel: one CTA per chunk.  It builds a 4096-entry decode table in shared memory for
//      each coded plane, then each warp decodes 4 sub-chunks (8 lanes each, one shared word stream
//      per sub-chunk), reads the raw planes of the same elements straight from the blob, merges
//      the planes, reverts the exponent bit reorder and writes the elements.  There is no planar
//      intermediate buffer.
// Every blob access is bounds-checked; a malformed unit raises a bit in the status word and its
// elements are zeroed.  No wait in these kernels depends on another thread's progress except
// __syncthreads().
#include <type_traits>
#include <vector>

#include "zn_common.cuh"

namespace zn {
namespace {

constexpr int kDecThreads = 128;  // 4 warps per chunk
constexpr int kChains = 1;        // rANS states per lane (sub-chunks per lane)
constexpr int kSym = 256 / kDecThreads;  // symbols per thread in table building
constexpr int64_t kCodedBit = int64_t(1) << 62;
constexpr int64_t kOffMask = kCodedBit - 1;

// One decompression job (a blob, or the payload list of the batched seam).  Jobs live in device
// memory; a decode CTA finds its job by global chunk index (find_job).
struct DecArgs {
  // whole-blob mode
  const uint8_t* blob;
  int64_t blob_bytes;
  int64_t* src;           // per unit: blob offset | kCodedBit, or -1 if invalid
  int64_t sizes_off, idx_off, data_off, n_comp;
  int64_t n, C, nch, units, chunk0;
  uint8_t* out;
  int32_t* status;
  // batched mode (K == 1): payload i at in_ptrs[i] (in_bytes[i]) decodes into out_ptrs[i]
  const int64_t* in_ptrs;
  const int64_t* in_bytes;
  const int64_t* out_ptrs;
  const int64_t* out_cap;
  int32_t* statuses;
  uint8_t* overflow;      // per chunk: more coded planes than the main pass holds
};

struct PlaneInfo {
  const uint8_t* pl;  // payload (coded) or raw bytes of this unit's chunk
  const uint8_t* lo;  // stream block loads may touch [lo, hi)
  const uint8_t* hi;
  int64_t size;
  int coded;
  int t;
  int single;              // the symbol of a plane with one symbol (f = M: no words, no state change), else -1
  int64_t states_off;
  int64_t lens_off;        // per-state stream lengths
  int lw;                  // bytes per length field
  int32_t stream_off[64];  // halfword index of each sub-chunk's first (lane 0) stream
};

struct DecSmem {
  uint32_t f[256];
  uint32_t cum[256];
  uint32_t red[8];
  int err;
  int t;
  PlaneInfo p[8];
};

__device__ __forceinline__ uint32_t block_sum(uint32_t v, uint32_t* red) {
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  uint32_t s = 0;
  for (int w = 0; w < kDecThreads / 32; ++w) s += red[w];
  return s;
}

__device__ __forceinline__ uint32_t block_excl(uint32_t v, uint32_t* red) {
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

// Parse a ZNR2 payload header and build its decode table.  Entry of slot z (symbol s, cum c, freq
// f < M): f << 20 | s << 12 | (z - c), so the state update f * (x >> 12) + (z - c) is one IMAD
// after the lookup.  A plane with a single symbol (f = M) needs no table: its state never changes
// and it has no words; P.single holds that symbol.  Returns false (uniformly) if the payload is
// malformed.
__device__ bool build_plane(PlaneInfo& P, int64_t m, uint32_t* tab, DecSmem& S) {
  const int tid = threadIdx.x;
  const uint8_t* pl = P.pl;
  const int64_t size = P.size;
  bool ok = size >= 34 && pl[0] >= kMinSubLog2 && pl[0] <= kMaxSubLog2 && pl[1] == 0;
  if (!__syncthreads_and(ok)) return false;
  const int t = pl[0];
  uint32_t pres[kSym], f4[kSym];
  uint32_t npres = 0;
#pragma unroll
  for (int h = 0; h < kSym; ++h) {
    const int s = kSym * tid + h;
    pres[h] = (pl[2 + (s >> 3)] >> (s & 7)) & 1;
    npres += pres[h];
  }
  const uint32_t np = block_sum(npres, S.red);
  const int64_t tb = table_bytes(int(np));
  const Geom g = geom_of(m, t);
  const int64_t mb = meta_bytes(int(np), g);
  if (np == 0 || mb > size) return false;
  uint32_t k = block_excl(npres, S.red);
  uint32_t fsum = 0;
#pragma unroll
  for (int h = 0; h < kSym; ++h) {
    f4[h] = 0;
    if (pres[h]) {
      const uint32_t bit = 12 * k++;
      const uint8_t* q = pl + 34 + (bit >> 3);
      const uint32_t v = (uint32_t(q[0]) | (uint32_t(q[1]) << 8) | (uint32_t(q[2]) << 16)) >> (bit & 7);
      f4[h] = (v & 0xFFF) + 1;
    }
    fsum += f4[h];
  }
  const uint32_t total = block_sum(fsum, S.red);
  if (total != kM) return false;
  if (np == 1) {
#pragma unroll
    for (int h = 0; h < kSym; ++h)
      if (pres[h]) P.single = kSym * tid + h;
  }
  uint32_t c0 = block_excl(fsum, S.red);
#pragma unroll
  for (int h = 0; h < kSym; ++h) {
    S.f[kSym * tid + h] = f4[h];
    S.cum[kSym * tid + h] = c0;
    c0 += f4[h];
  }
  // Per-sub-chunk stream offsets (sum of its 8 lane lengths; one warp, one sub-chunk per lane).
  if (tid < 32) {
    int64_t pos = mb / 2;
    bool good = true;
    for (int g0 = 0; g0 < g.nu; g0 += 32) {
      const int gi = g0 + tid;
      int64_t sub = 0;
      if (gi < g.nu)
        for (int l = 0; l < kLanes; ++l) {
          const int64_t fi = int64_t(gi) * kLanes + l;
          const int64_t nw = g.lw == 2 ? int64_t(pl[tb + 2 * fi]) | (int64_t(pl[tb + 2 * fi + 1]) << 8)
                                       : int64_t(*reinterpret_cast<const uint32_t*>(pl + tb + 4 * fi));
          good &= nw <= g.sc / kLanes;
          sub += nw;
        }
      int64_t incl = sub;
      for (int o = 1; o < 32; o <<= 1) {
        const int64_t v = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (tid >= o) incl += v;
      }
      if (gi < g.nu) P.stream_off[gi] = int32_t(pos + incl - sub);
      pos += __shfl_sync(0xFFFFFFFFu, incl, 31);
    }
    good = __all_sync(0xFFFFFFFFu, good);
    if (tid == 0) {
      P.t = t;
      P.lens_off = tb;
      P.lw = g.lw;
      P.states_off = tb + lengths_bytes(g);
      S.err = !(good && 2 * pos == size);
    }
  }
  __syncthreads();
  if (S.err) return false;
  // Fill the slot table, one symbol per warp iteration, 32 slots per step.
  const int lane = tid & 31, warp = tid >> 5;
  for (int s = warp; s < 256; s += kDecThreads / 32) {
    const uint32_t f = S.f[s], c = S.cum[s];
    const uint32_t hi = (f << 20) | (uint32_t(s) << 12);  // f = M (one symbol) wraps: the table is unused
    for (uint32_t q = lane; q < f; q += 32) tab[c + q] = hi | q;
  }
  __syncthreads();
  return true;
}

// One 16-byte block of a word stream.  Blocks wholly inside [lo, hi) are one 16-byte load; a block
// that straddles the edge is read halfword by halfword (outside halfwords read as 0).
__device__ __forceinline__ uint4 load_block(const uint8_t* gb, uint32_t q, const uint8_t* lo, const uint8_t* hi) {
  const uint8_t* p = gb + 16 * uint64_t(q);
  if (p >= lo && p + 16 <= hi) return __ldg(reinterpret_cast<const uint4*>(p));
  uint32_t w[4] = {0, 0, 0, 0};
#pragma unroll
  for (int h = 0; h < 8; ++h) {
    const uint8_t* q2 = p + 2 * h;
    if (q2 >= lo && q2 + 2 <= hi) w[h >> 1] |= uint32_t(*reinterpret_cast<const uint16_t*>(q2)) << (16 * (h & 1));
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Decoder state of one rANS state (a lane of a sub-chunk) of one coded plane.  Stream positions
// are halfword indices relative to the 16-byte aligned base gb of the payload.  Each state keeps
// a ring of kRing words of its stream in shared memory: at every round start [ptr, ptr + 16) is
// present (a round consumes at most 16 words) and 16-byte blocks ahead are loaded, to be stored
// at the round's end.
struct Cursor {
  uint32_t x, ptr, end, fill, nload;
  uint4 r0, r1;
};

// Ring layout: slot p of the state of thread t sits at rings[(p % kRing) * kDecThreads + t] (rows
// of kDecThreads slots), so the 32 states of a warp read their next words from 32 different banks
// when a slot is 32 bits wide (one stream halfword in its low half; the decoder ignores the upper
// half).  With more than 4 coded planes in shared memory the slots are halfwords (at most two
// lanes per bank).
constexpr int kRing = 32;
template <int KC>
using RingSlot = std::conditional_t<(KC > 4), uint16_t, uint32_t>;

// Store the 16-byte stream block that starts at halfword `fill` (a multiple of 8) into a ring.
template <typename Slot>
__device__ __forceinline__ void ring_put(Slot* ring, uint32_t fill, const uint4& v) {
  Slot* r = ring + (fill & (kRing - 1)) * kDecThreads;
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    r[(2 * i) * kDecThreads] = Slot(w[i]);
    r[(2 * i + 1) * kDecThreads] = Slot(w[i] >> 16);
  }
}

// One decode step of one state (symbol into byte (i & 3) of acc, next word read one step ahead).
template <bool FULL, int I, typename Slot>
__device__ __forceinline__ void decode_step(uint32_t& xv, uint32_t& pv, uint32_t& wn, uint32_t& acc, bool act,
                                            const uint32_t* __restrict__ tab, const Slot* ring) {
  const uint32_t e = tab[xv & (kM - 1)];
  const uint32_t q = xv >> kScaleBits;
  uint32_t xn = (e >> 20) * q + (e & 0xFFFu);
  if (!FULL) xn = act ? xn : xv;
  acc = __byte_perm(acc, e >> 12, (0x3210 & ~(0xF << (4 * (I & 3)))) | (4 << (4 * (I & 3))));
  const bool need = (FULL || act) && xn < kL;
  const uint32_t w = wn;
  pv += need;
  wn = ring[(pv & (kRing - 1)) * kDecThreads];
  xv = need ? __byte_perm(w, xn, 0x5410) : xn;  // (xn << 16) | (w & 0xFFFF)
}

// 16 steps of the lane's kChains states, interleaved so the independent chains overlap.  A stream
// over-read is not tested per step: it leaves the final state or position wrong, which the caller
// checks (ring reads are always in bounds).
template <bool FULL, typename Slot>
__device__ __forceinline__ void decode_round(Cursor* cb, const uint32_t* __restrict__ tab, Slot* const* ring,
                                             const int* nact, uint32_t (*acc)[4]) {
  uint32_t xv[kChains], pv[kChains], wn[kChains];
#pragma unroll
  for (int c = 0; c < kChains; ++c) {
    xv[c] = cb[c].x;
    pv[c] = cb[c].ptr;
    wn[c] = ring[c][(pv[c] & (kRing - 1)) * kDecThreads];
  }
#define ZN_STEP(I)                                                                                    \
  _Pragma("unroll") for (int c = 0; c < kChains; ++c)                                                 \
      decode_step<FULL, I>(xv[c], pv[c], wn[c], acc[c][(I) >> 2], (I) < nact[c], tab, ring[c]);
  ZN_STEP(0) ZN_STEP(1) ZN_STEP(2) ZN_STEP(3) ZN_STEP(4) ZN_STEP(5) ZN_STEP(6) ZN_STEP(7)
  ZN_STEP(8) ZN_STEP(9) ZN_STEP(10) ZN_STEP(11) ZN_STEP(12) ZN_STEP(13) ZN_STEP(14) ZN_STEP(15)
#undef ZN_STEP
#pragma unroll
  for (int c = 0; c < kChains; ++c) {
    cb[c].x = xv[c];
    cb[c].ptr = pv[c];
  }
}

// The fast path's 16 steps of the lane's kChains states.  A state's ring position is kept as the
// byte offset tid * 4 + (ptr % kRing) * kDecThreads * 4 from its ring's first row, so the word
// read after a renormalisation costs one masked add; the position advance is recovered at the end
// (a round consumes at most 16 < kRing words).
__device__ __forceinline__ void decode_round_fast(Cursor* cb, const uint32_t* __restrict__ tab, const uint8_t* rows,
                                                  int tid, uint32_t (*acc)[4]) {
  constexpr uint32_t kRowBytes = kDecThreads * 4, kRingBytes = kRing * kRowBytes;
  uint32_t xv[kChains], ro[kChains], ro0[kChains], wn[kChains];
#pragma unroll
  for (int c = 0; c < kChains; ++c) {
    xv[c] = cb[c].x;
    ro0[c] = uint32_t(tid) * 4 + (cb[c].ptr & (kRing - 1)) * kRowBytes;
    ro[c] = ro0[c];
    wn[c] = *reinterpret_cast<const uint32_t*>(rows + c * kRingBytes + ro[c]);
  }
#define ZN_FSTEP(I)                                                                                   \
  _Pragma("unroll") for (int c = 0; c < kChains; ++c) {                                               \
    const uint32_t e = tab[xv[c] & (kM - 1)];                                                         \
    const uint32_t xn = (e >> 20) * (xv[c] >> kScaleBits) + (e & 0xFFFu);                             \
    acc[c][(I) >> 2] = __byte_perm(acc[c][(I) >> 2], e >> 12,                                         \
                                   (0x3210 & ~(0xF << (4 * ((I) & 3)))) | (4 << (4 * ((I) & 3))));    \
    const bool need = xn < kL;                                                                        \
    const uint32_t w = wn[c];                                                                         \
    ro[c] = need ? ((ro[c] + kRowBytes) & (kRingBytes - 1)) : ro[c];                                  \
    wn[c] = *reinterpret_cast<const uint32_t*>(rows + c * kRingBytes + ro[c]);                        \
    xv[c] = need ? __byte_perm(w, xn, 0x5410) : xn;                                                   \
  }
  ZN_FSTEP(0) ZN_FSTEP(1) ZN_FSTEP(2) ZN_FSTEP(3) ZN_FSTEP(4) ZN_FSTEP(5) ZN_FSTEP(6) ZN_FSTEP(7)
  ZN_FSTEP(8) ZN_FSTEP(9) ZN_FSTEP(10) ZN_FSTEP(11) ZN_FSTEP(12) ZN_FSTEP(13) ZN_FSTEP(14) ZN_FSTEP(15)
#undef ZN_FSTEP
#pragma unroll
  for (int c = 0; c < kChains; ++c) {
    cb[c].x = xv[c];
    cb[c].ptr += (ro[c] / kRowBytes - ro0[c] / kRowBytes) & (kRing - 1);
  }
}

// The 16 symbols of a round of a one-symbol plane, for every chain.
__device__ __forceinline__ void fill_single(uint32_t (*acc)[4], int s) {
#pragma unroll
  for (int c = 0; c < kChains; ++c)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[c][i] = uint32_t(s) * 0x01010101u;
}

// Raw (stored) plane bytes of round r for each chain: 16 bytes per plane from the lane's 16
// symbols, byte by byte in a partial last round.  Coded planes are left untouched.
template <int K, int NC>
__device__ __forceinline__ void load_raw_round(const uint8_t* const* src, const bool* coded, const int64_t* base,
                                               const int64_t* len, int r, int l, uint32_t (*p)[K][4]) {
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int64_t off = int64_t(r) * kRound + l * kSteps;
    const int nact = int(max(int64_t(0), min(int64_t(kSteps), len[c] - off)));
#pragma unroll
    for (int b = 0; b < K; ++b) {
      if (coded[b]) continue;
      const uint8_t* sp = src[b] + base[c] + off;
      if (nact == 16) {
        const uint2 v0 = reinterpret_cast<const uint2*>(sp)[0], v1 = reinterpret_cast<const uint2*>(sp)[1];
        p[c][b][0] = v0.x; p[c][b][1] = v0.y; p[c][b][2] = v1.x; p[c][b][3] = v1.y;
      } else {
        uint64_t vlo = 0, vhi = 0;
        for (int i = 0; i < nact; ++i) {
          const uint64_t byte = sp[i];
          if (i < 8) vlo |= byte << (8 * i);
          else vhi |= byte << (8 * (i - 8));
        }
        p[c][b][0] = uint32_t(vlo); p[c][b][1] = uint32_t(vlo >> 32);
        p[c][b][2] = uint32_t(vhi); p[c][b][3] = uint32_t(vhi >> 32);
      }
    }
  }
}

// 16 elements (4 * K little-endian words) from their K byte planes (4 words each), with the
// exponent reorder undone.  bf16 has a direct form: with E the exponent plane (high bytes after
// the reorder, e8) and B the sign / mantissa plane (s m7), the element's high byte is
// s | e8 >> 1 and its low byte (e8 & 1) << 7 | m7, four elements per 32-bit operation.
template <int K, bool REORDER>
__device__ __forceinline__ void assemble_elements(const uint32_t (*p)[4], uint32_t* e) {
  if constexpr (K == 2 && REORDER) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t E = p[1][i], B = p[0][i];
      const uint32_t hi = (B & 0x80808080u) | ((E >> 1) & 0x7F7F7F7Fu);
      const uint32_t lo = ((E << 7) & 0x80808080u) | (B & 0x7F7F7F7Fu);
      e[2 * i] = __byte_perm(lo, hi, 0x5140);
      e[2 * i + 1] = __byte_perm(lo, hi, 0x7362);
    }
  } else {
    planes_to_elements<K>(p, e);
    reorder_words<K, REORDER, false>(e, 4 * K);
  }
}

// Decode global chunk gchunk with the whole CTA.  KC: coded planes per chunk held in shared
// memory.  The main pass (KC = 1 for K > 1) flags chunks with more coded planes; a second pass
// with KC = K decodes only those.  Every return is taken by all threads of the CTA together.
// Work split: a warp item is 8 sub-chunks; lane l of 8-lane segment g runs chain c on sub-chunk
// 8 * item + 4 * c + g.
template <int K, bool REORDER, int KC>
__device__ __forceinline__ void decode_chunk(const DecArgs* __restrict__ jobs, int njobs, int64_t gchunk,
                                             bool overflow_pass) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  using Slot = RingSlot<KC>;
  uint32_t* tabs = reinterpret_cast<uint32_t*>(smem_raw);                      // [KC][4096]
  Slot* rings = reinterpret_cast<Slot*>(smem_raw + KC * kM * 4);                // [KC][kChains][kRing][threads]
  DecSmem& S = *reinterpret_cast<DecSmem*>(smem_raw + KC * kM * 4 + KC * kChains * kRing * kDecThreads * sizeof(Slot));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const DecArgs& a = jobs[find_job(jobs, njobs, gchunk)];
  const int64_t j = gchunk - a.chunk0;
  if (overflow_pass && !a.overflow[j]) return;
  const bool batched = a.in_ptrs != nullptr;
  int64_t m;
  uint8_t* outc;
  if (batched) {
    m = a.out_cap[j];
    outc = reinterpret_cast<uint8_t*>(a.out_ptrs[j]);
  } else {
    m = min(a.C, a.n - j * a.C);
    outc = a.out + j * a.C * K;
  }
  if (tid == 0) S.err = 0;
  if (tid < K) {
    PlaneInfo& P = S.p[tid];
    if (batched) {
      P.pl = reinterpret_cast<const uint8_t*>(a.in_ptrs[j]);
      P.size = a.in_bytes[j];
      P.coded = 1;
      P.lo = P.pl;
      P.hi = P.pl + P.size;
    } else {
      const int64_t u = int64_t(tid) * a.nch + j;
      const int64_t s = a.src[u];
      // dscan_kernel has checked that the tables lie inside the blob for every unit with s >= 0.
      const int64_t stored = s >= 0 ? *reinterpret_cast<const int32_t*>(a.blob + a.sizes_off + 4 * u) : 0;
      P.coded = s >= 0 && (s & kCodedBit);
      P.pl = a.blob + (s & kOffMask);
      P.size = stored;
      P.lo = a.blob;
      P.hi = a.blob + a.blob_bytes;
      if (s < 0) atomicOr(&S.err, 1);
    }
    P.t = -1;
    P.single = -1;
  }
  __syncthreads();
  int ncoded = 0;
  int pslot[KC];  // plane of each coded slot
#pragma unroll
  for (int q = 0; q < KC; ++q) pslot[q] = 0;
  for (int b = 0; b < K; ++b)
    if (S.p[b].coded) {
      if (ncoded < KC) pslot[ncoded] = b;
      ++ncoded;
    }
  if (KC < K && !overflow_pass) {
    const bool over = ncoded > KC;
    if (tid == 0) a.overflow[j] = over;
    if (over) return;
  }
  bool bad = S.err != 0 || m <= 0;
  for (int q = 0; q < KC && q < ncoded && !bad; ++q)
    if (!build_plane(S.p[pslot[q]], m, tabs + q * kM, S)) bad = true;
  int t = 4;
  if (!bad && ncoded) {
    t = S.p[pslot[0]].t;
    // All coded planes of a chunk must share one sub-chunk geometry.
    for (int q = 0; q < KC && q < ncoded; ++q)
      if (S.p[pslot[q]].t != t) bad = true;
  }
  if (bad) {
    if (tid == 0) {
      if (batched) a.statuses[j] = kErrPayload;
      else atomicOr(a.status, kErrPayload);
    }
    if (m > 0)
      for (int64_t i = tid; i < m * K; i += kDecThreads) outc[i] = 0;
    return;
  }

  const Geom g = geom_of(m, t);
  const int seg = lane >> 3, l = lane & 7;
  const int rounds = int(g.sc / kRound);
  const bool out16 = (reinterpret_cast<uintptr_t>(outc) & 15) == 0;
  bool coded[K];
  const uint8_t* src[K];
#pragma unroll
  for (int b = 0; b < K; ++b) {
    coded[b] = S.p[b].coded;
    src[b] = S.p[b].pl;
  }
  const uint8_t* gb[KC];
  const uint8_t* lo[KC];
  const uint8_t* hi[KC];
#pragma unroll
  for (int q = 0; q < KC; ++q) {
    gb[q] = reinterpret_cast<const uint8_t*>(reinterpret_cast<uintptr_t>(S.p[pslot[q]].pl) & ~uintptr_t(15));
    lo[q] = S.p[pslot[q]].lo;
    hi[q] = S.p[pslot[q]].hi;
  }
  bool err = false;
  const int items = int(cdiv(g.nu, 4 * kChains));
  for (int item = warp; item < items; item += kDecThreads / 32) {
    int gi[kChains];
    int64_t base[kChains], len[kChains];
    bool valid[kChains];
#pragma unroll
    for (int c = 0; c < kChains; ++c) {
      gi[c] = 4 * kChains * item + 4 * c + seg;
      valid[c] = gi[c] < g.nu;
      base[c] = int64_t(gi[c]) * g.sc;
      len[c] = valid[c] ? min(g.sc, m - base[c]) : 0;
    }
    Cursor cur[KC][kChains];
    Slot* ring[KC][kChains];
    int single[KC];  // symbol of a one-symbol coded plane, else -1
#pragma unroll
    for (int q = 0; q < KC; ++q) single[q] = q < ncoded ? S.p[pslot[q]].single : -1;
#pragma unroll
    for (int q = 0; q < KC; ++q)
#pragma unroll
      for (int c = 0; c < kChains; ++c) {
        Cursor& cb = cur[q][c];
        ring[q][c] = rings + (q * kChains + c) * kRing * kDecThreads + tid;
        cb.x = kL;
        cb.ptr = cb.end = cb.fill = cb.nload = 0;
        if (q < ncoded && valid[c]) {
          const PlaneInfo& P = S.p[pslot[q]];
          const int64_t fbase = int64_t(gi[c]) * kLanes;
          uint32_t before = 0, mine = 0;
          for (int ll = 0; ll <= l; ++ll) {
            const int64_t fi = fbase + ll;
            const uint32_t nw = P.lw == 2 ? *reinterpret_cast<const uint16_t*>(P.pl + P.lens_off + 2 * fi)
                                          : *reinterpret_cast<const uint32_t*>(P.pl + P.lens_off + 4 * fi);
            if (ll < l) before += nw;
            else mine = nw;
          }
          const uint32_t h0 = uint32_t((P.pl - gb[q]) >> 1) + uint32_t(P.stream_off[gi[c]]) + before;
          cb.x = *reinterpret_cast<const uint32_t*>(P.pl + P.states_off + 4 * (fbase + l));
          cb.ptr = h0;
          cb.end = h0 + mine;
          cb.fill = h0 & ~7u;
          err |= cb.x < kL || cb.x >= 0x80000000u;
        }
      }
    uint32_t pn[kChains][K][4];
    load_raw_round<K, kChains>(src, coded, base, len, 0, l, pn);
    int r = 0;
    if constexpr (KC == 1) {
      // Full rounds (all 16 steps of every chain's state valid): no per-step predication, 32-bit
      // bookkeeping and running element offsets; the partial rounds at the end of a sub-chunk
      // take the general loop below.
      const int64_t l16 = int64_t(l) * kSteps;
      int rfull = rounds;
      uint32_t end8[kChains], off[kChains];  // off: element offset of the lane's round r in the chunk
#pragma unroll
      for (int c = 0; c < kChains; ++c) {
        rfull = min(rfull, len[c] >= l16 + kSteps ? int((len[c] - l16 - kSteps) / kRound) + 1 : 0);
        end8[c] = (cur[0][c].end + 7) & ~7u;
        off[c] = uint32_t(base[c] + l16);
      }
      // Stream blocks [qbeg, qend) from gb lie wholly inside [lo, hi): one 16-byte load each.
      const uint4* gb4 = reinterpret_cast<const uint4*>(gb[0]);
      const uint32_t qbeg = gb[0] < lo[0] ? 1u : 0u;
      const uint64_t span = hi[0] > gb[0] ? uint64_t(hi[0] - gb[0]) / 16 : 0;
      const uint32_t qend = span > 0xFFFFFFFFull ? 0xFFFFFFFFu : uint32_t(span);
      auto block = [&](uint32_t q) {
        return q >= qbeg && q < qend ? __ldg(gb4 + q) : load_block(gb[0], q, lo[0], hi[0]);
      };
      const uint8_t* rows = reinterpret_cast<const uint8_t*>(rings);
      // LAST: the one coded plane is plane K - 1 (the exponent plane of every float type), so the
      // raw planes and the decoded symbols have fixed places (no per-round plane selection).
      auto full_rounds = [&](auto last) {
        constexpr bool LAST = decltype(last)::value;
        for (; r < rfull; ++r) {
          if (LAST || ncoded > 0) {
            // [ptr, ptr + 16) must be present (synchronous loads only when the ring ran low), then
            // at most one block is fetched ahead per round, stored at the round's end.
#pragma unroll
            for (int c = 0; c < kChains; ++c) {
              Cursor& cb = cur[0][c];
              const uint32_t need = min((cb.ptr + 16 + 7) & ~7u, end8[c]);
              while (cb.fill < need) {
                ring_put(ring[0][c], cb.fill, block(cb.fill / 8));
                cb.fill += 8;
              }
              cb.nload = cb.fill < end8[c] && cb.fill + 8 <= cb.ptr + kRing ? 1u : 0u;
              if (cb.nload) cb.r0 = block(cb.fill / 8);
            }
          }
          uint32_t p[kChains][K][4];
#pragma unroll
          for (int c = 0; c < kChains; ++c)
#pragma unroll
            for (int b = 0; b < K; ++b)
#pragma unroll
              for (int i = 0; i < 4; ++i) p[c][b][i] = pn[c][b][i];
          if (r + 1 < rfull) {
#pragma unroll
            for (int c = 0; c < kChains; ++c)
#pragma unroll
              for (int b = 0; b < K; ++b) {
                if (LAST ? b == K - 1 : coded[b]) continue;
                const uint2* sp = reinterpret_cast<const uint2*>(src[b] + off[c] + kRound);
                const uint2 v0 = sp[0], v1 = sp[1];
                pn[c][b][0] = v0.x; pn[c][b][1] = v0.y; pn[c][b][2] = v1.x; pn[c][b][3] = v1.y;
              }
          } else if (r + 1 < rounds) {
            load_raw_round<K, kChains>(src, coded, base, len, r + 1, l, pn);
          }
          if (LAST || ncoded > 0) {
            uint32_t acc[kChains][4] = {};
            if (single[0] < 0) decode_round_fast(cur[0], tabs, rows, tid, acc);
            else fill_single(acc, single[0]);
#pragma unroll
            for (int c = 0; c < kChains; ++c) {
#pragma unroll
              for (int b = 0; b < K; ++b)
                if (LAST ? b == K - 1 : b == pslot[0]) {
#pragma unroll
                  for (int i = 0; i < 4; ++i) p[c][b][i] = acc[c][i];
                }
              Cursor& cb = cur[0][c];
              if (cb.nload) ring_put(ring[0][c], cb.fill, cb.r0);
              cb.fill += 8 * cb.nload;
            }
          }
#pragma unroll
          for (int c = 0; c < kChains; ++c) {
            uint32_t e[4 * K];
            assemble_elements<K, REORDER>(p[c], e);
            store_words(outc + size_t(off[c]) * K, e, 4 * K, out16);  // 16-byte aligned when outc is
            off[c] += kRound;
          }
        }
      };
      if (ncoded == 1 && pslot[0] == K - 1) full_rounds(std::true_type{});
      else full_rounds(std::false_type{});
    }
    for (; r < rounds; ++r) {
      int nact[kChains];
      int64_t off[kChains];
#pragma unroll
      for (int c = 0; c < kChains; ++c) {
        off[c] = int64_t(r) * kRound + l * kSteps;
        nact[c] = int(max(int64_t(0), min(int64_t(kSteps), len[c] - off[c])));
      }
      // Ring upkeep: make [ptr, ptr + 16) present, start up to two block loads ahead.
#pragma unroll
      for (int q = 0; q < KC; ++q) {
        if (q >= ncoded) break;
#pragma unroll
        for (int c = 0; c < kChains; ++c) {
          Cursor& cb = cur[q][c];
          const uint32_t end8 = (cb.end + 7) & ~7u;
          const uint32_t need = min((cb.ptr + 16 + 7) & ~7u, end8);
          while (cb.fill < need) {
            ring_put(ring[q][c], cb.fill, load_block(gb[q], cb.fill / 8, lo[q], hi[q]));
            cb.fill += 8;
          }
          const uint32_t limit = min((cb.ptr + kRing) & ~7u, end8);
          cb.nload = limit > cb.fill ? min((limit - cb.fill) / 8, 2u) : 0u;
          if (cb.nload > 0) cb.r0 = load_block(gb[q], cb.fill / 8, lo[q], hi[q]);
          if (cb.nload > 1) cb.r1 = load_block(gb[q], cb.fill / 8 + 1, lo[q], hi[q]);
        }
      }
      // This round's raw-plane bytes were loaded during the previous round; start the next
      // round's loads now, so that they overlap this round's decoding.
      uint32_t p[kChains][K][4];
#pragma unroll
      for (int c = 0; c < kChains; ++c)
#pragma unroll
        for (int b = 0; b < K; ++b)
#pragma unroll
          for (int i = 0; i < 4; ++i) p[c][b][i] = pn[c][b][i];
      if (r + 1 < rounds) load_raw_round<K, kChains>(src, coded, base, len, r + 1, l, pn);
      const bool full = nact[0] == kSteps && nact[kChains - 1] == kSteps;
#pragma unroll
      for (int q = 0; q < KC; ++q) {
        if (q >= ncoded) break;
        uint32_t acc[kChains][4] = {};
        if (single[q] >= 0) fill_single(acc, single[q]);
        else if (full) decode_round<true>(cur[q], tabs + q * kM, ring[q], nact, acc);
        else decode_round<false>(cur[q], tabs + q * kM, ring[q], nact, acc);
#pragma unroll
        for (int c = 0; c < kChains; ++c)
#pragma unroll
          for (int b = 0; b < K; ++b)
            if (b == pslot[q]) {
#pragma unroll
              for (int i = 0; i < 4; ++i) p[c][b][i] = acc[c][i];
            }
      }
      // Store the blocks loaded at the round's start (this round's reads are done).
#pragma unroll
      for (int q = 0; q < KC; ++q) {
        if (q >= ncoded) break;
#pragma unroll
        for (int c = 0; c < kChains; ++c) {
          Cursor& cb = cur[q][c];
          if (cb.nload > 0) ring_put(ring[q][c], cb.fill, cb.r0);
          if (cb.nload > 1) ring_put(ring[q][c], cb.fill + 8, cb.r1);
          cb.fill += 8 * cb.nload;
        }
      }
#pragma unroll
      for (int c = 0; c < kChains; ++c) {
        if (nact[c] <= 0) continue;
        uint32_t e[4 * K];
        assemble_elements<K, REORDER>(p[c], e);
        uint8_t* dst = outc + (base[c] + off[c]) * K;
        if (nact[c] == 16) {
          store_words(dst, e, 4 * K, out16 && ((((base[c] + off[c]) * K) & 15) == 0));
        } else {
#pragma unroll
          for (int w = 0; w < 4 * K; ++w)
#pragma unroll
            for (int qq = 0; qq < 4; ++qq)
              if (4 * w + qq < nact[c] * K) dst[4 * w + qq] = uint8_t(e[w] >> (8 * qq));
        }
      }
    }
#pragma unroll
    for (int q = 0; q < KC; ++q)
#pragma unroll
      for (int c = 0; c < kChains; ++c)
        if (q < ncoded && valid[c]) err |= (cur[q][c].x != kL) || (cur[q][c].ptr != cur[q][c].end);
  }
  if (__syncthreads_or(err) && tid == 0) {
    if (batched) a.statuses[j] = kErrStream;
    else atomicOr(a.status, kErrStream);
  } else if (batched && tid == 0) {
    a.statuses[j] = 0;
  }
}

// Main pass: one CTA per chunk.
template <int K, bool REORDER, int KC>
__global__ void __launch_bounds__(kDecThreads) decode_kernel(const DecArgs* __restrict__ jobs, int njobs) {
  decode_chunk<K, REORDER, KC>(jobs, njobs, blockIdx.x, false);
}

// Overflow pass: a grid of resident CTAs scans the per-chunk flags, kDecThreads chunks a round at a
// stride of the grid (flagged chunks that cluster in one tensor spread over the CTAs), and decodes
// the flagged ones one after another.
template <int K, bool REORDER, int KC>
__global__ void __launch_bounds__(kDecThreads) decode_overflow_kernel(const DecArgs* __restrict__ jobs, int njobs,
                                                                      int64_t total_chunks) {
  __shared__ int64_t flagged[kDecThreads];
  __shared__ int nflagged;
  const int64_t stride = gridDim.x;
  for (int64_t first = blockIdx.x; first < total_chunks; first += stride * kDecThreads) {
    const int64_t c = first + stride * threadIdx.x;
    bool f = false;
    if (c < total_chunks) {
      const DecArgs& a = jobs[find_job(jobs, njobs, c)];
      f = a.overflow[c - a.chunk0] != 0;
    }
    if (threadIdx.x == 0) nflagged = 0;
    __syncthreads();
    if (f) flagged[atomicAdd(&nflagged, 1)] = c;
    __syncthreads();
    const int nf = nflagged;
    for (int q = 0; q < nf; ++q) {
      decode_chunk<K, REORDER, KC>(jobs, njobs, flagged[q], true);
      __syncthreads();
    }
    __syncthreads();
  }
}

// ---- table scan (src/cuzipnn/_codec.py:492-496, 529) ----------------------------------------

constexpr int kScanThreads = 1024;

// One CTA per job.  It first zeroes the job's status word.  A job whose n_comp is negative reads
// it from the blob's header (u32 at byte 12) here; tables that do not fit the blob then mark every
// unit invalid (the decoder zero-fills them) and set kErrTable.
// The first kernel of a call: a single-job call passes its job by value (`one`), which CTA 0 also
// stores into the table at `table` for the kernels after this one.
__global__ void __launch_bounds__(kScanThreads) dscan_kernel(const DecArgs* __restrict__ jobs,
                                                             const __grid_constant__ FirstJob<DecArgs> one,
                                                             DecArgs* table) {
  __shared__ int64_t sm[64];
  __shared__ int64_t s_ncomp;
  if (one.valid && blockIdx.x == 0) store_job(one.job, table);
  const DecArgs& a = one.valid ? one.job : jobs[blockIdx.x];
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  if (tid == 0) {
    *a.status = 0;
    int64_t nc = a.n_comp;
    if (nc < 0) nc = a.blob_bytes >= 16 ? int64_t(*reinterpret_cast<const uint32_t*>(a.blob + 12)) : -1;
    s_ncomp = nc;
  }
  __syncthreads();
  const int64_t n_comp = s_ncomp;
  const int64_t data_off = align8(a.idx_off + 4 * n_comp);
  if (n_comp < 0 || n_comp > a.units || data_off > a.blob_bytes) {
    for (int64_t i = tid; i < a.units; i += kScanThreads) a.src[i] = -1;
    if (tid == 0) atomicOr(a.status, kErrTable);
    return;
  }
  const int64_t last = a.n - (a.nch - 1) * a.C;
  const int32_t* stored = reinterpret_cast<const int32_t*>(a.blob + a.sizes_off);
  int64_t carry = data_off;
  bool bad = false;
  for (int64_t start = 0; start < a.units; start += kScanThreads) {
    const int64_t i = start + tid;
    int64_t v = 0;
    if (i < a.units) {
      const int64_t s = stored[i];
      bad |= s < 0;
      v = s < 0 ? 0 : align8(s);
    }
    int64_t incl = v;
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t u = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += u;
    }
    if (lane == 31) sm[w] = incl;
    __syncthreads();
    if (w == 0) {
      int64_t q = sm[lane];
      for (int o = 1; o < 32; o <<= 1) {
        const int64_t u = __shfl_up_sync(0xFFFFFFFFu, q, o);
        if (lane >= o) q += u;
      }
      sm[32 + lane] = q;
    }
    __syncthreads();
    const int64_t excl = carry + (w ? sm[32 + w - 1] : 0) + incl - v;
    if (i < a.units) a.src[i] = excl;
    carry += sm[32 + 31];
    __syncthreads();
  }
  __syncthreads();
  const int32_t* idx = reinterpret_cast<const int32_t*>(a.blob + a.idx_off);
  for (int64_t q = tid; q < n_comp; q += kScanThreads) {
    const int64_t i = idx[q];
    if (i < 0 || i >= a.units) { bad = true; continue; }
    a.src[i] |= kCodedBit;
  }
  __syncthreads();
  for (int64_t i = tid; i < a.units; i += kScanThreads) {
    const int64_t s = a.src[i];
    const int64_t off = s & kOffMask, st = stored[i];
    const int64_t raw = (i % a.nch) == a.nch - 1 ? last : a.C;
    const bool coded = s & kCodedBit;
    // A raw unit holds exactly the chunk's bytes; a coded one must lie inside the blob.
    if (st < 0 || off + st > a.blob_bytes || (!coded && st != raw)) {
      a.src[i] = -1;
      bad = true;
    }
  }
  if (__syncthreads_or(bad) && tid == 0) atomicOr(a.status, kErrTable);
}

size_t dec_smem(int KC) {
  return size_t(KC) * kM * 4 + size_t(KC) * kChains * kRing * kDecThreads * (KC > 4 ? 2 : 4) + sizeof(DecSmem);
}

template <int K, bool REORDER, int KC, bool OVERFLOW>
int launch_decode_pass(const DecArgs* jobs, int njobs, int64_t total_chunks, cudaStream_t s) {
  const size_t sm = dec_smem(KC);
  if constexpr (!OVERFLOW) {
    auto fn = decode_kernel<K, REORDER, KC>;
    if (int rc = set_max_smem(reinterpret_cast<const void*>(fn), int(sm))) return rc;
    TimedLaunch tl("decode", s);
    fn<<<unsigned(total_chunks), kDecThreads, sm, s>>>(jobs, njobs);
  } else {
    auto fn = decode_overflow_kernel<K, REORDER, KC>;
    if (int rc = set_max_smem(reinterpret_cast<const void*>(fn), int(sm))) return rc;
    int dev = 0, sms = 0, per_sm = 0;  // the grid: the CTAs that fit on the device at once
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kDecThreads, sm);
    if (e != cudaSuccess) return set_error(ZN_ERR_CUDA, "decode_overflow_kernel occupancy: %s", cudaGetErrorString(e));
    const int64_t grid = min(total_chunks, int64_t(max(1, sms * per_sm)));
    TimedLaunch tl("decode_overflow", s);
    fn<<<unsigned(grid), kDecThreads, sm, s>>>(jobs, njobs, total_chunks);
  }
  count_launch();
  return check_launch("decode_kernel");
}

// Main pass with one coded plane per chunk in shared memory, then (K > 1) the overflow pass.
template <int K, bool REORDER>
int launch_decode(const DecArgs* jobs, int njobs, int64_t grid, cudaStream_t s) {
  if (grid <= 0) return ZN_OK;
  if (int rc = launch_decode_pass<K, REORDER, 1, false>(jobs, njobs, grid, s)) return rc;
  if constexpr (K > 1) return launch_decode_pass<K, REORDER, K, true>(jobs, njobs, grid, s);
  return ZN_OK;
}

size_t dec_job_bytes(int64_t n, int k, int64_t chunk_bytes) {
  const int64_t nch = cdiv(n, chunk_bytes);
  return (size_t(int64_t(k) * nch) * 8 + size_t(nch) + 255) & ~size_t(255);  // unit offsets, overflow flags
}

}  // namespace
}  // namespace zn

using namespace zn;

extern "C" {

size_t zn_ans_decompress_temp_bytes(int64_t count) { return job_table_bytes<DecArgs>(1, count); }

int zn_ans_decompress(const int64_t* in_ptrs, const int64_t* in_bytes, const int64_t* out_capacity, int64_t count,
                      const int64_t* out_ptrs, int32_t* statuses, void* temp, size_t temp_bytes, void* stream) {
  if (count < 0 || count > 0x7FFFFFFF) return set_error(ZN_ERR_INVALID, "zn_ans_decompress: bad arguments");
  if (count == 0) return ZN_OK;
  if (!temp || temp_bytes < job_table_bytes<DecArgs>(1, count)) return set_error(ZN_ERR_SPACE, "zn_ans_decompress: temp buffer too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  DecArgs a{};
  a.in_ptrs = in_ptrs;
  a.in_bytes = in_bytes;
  a.out_ptrs = out_ptrs;
  a.out_cap = out_capacity;
  a.statuses = statuses;
  a.nch = count;
  DecArgs* dj = static_cast<DecArgs*>(temp);
  if (int rc = upload_jobs(&a, 1, dj, count, s)) return rc;
  return launch_decode<1, false>(dj, 1, count, s);
}

size_t zn_decompress_batch_temp_bytes(int njobs, const int64_t* n, int k, const int64_t* chunk_bytes) {
  if (njobs < 0 || k <= 0) return 0;
  size_t total = 0;
  int64_t chunks = 0;
  for (int i = 0; i < njobs; ++i) {
    if (n[i] < 0 || chunk_bytes[i] <= 0) return 0;
    chunks += cdiv(n[i], chunk_bytes[i]);
    total += dec_job_bytes(n[i], k, chunk_bytes[i]);
  }
  return total + job_table_bytes<DecArgs>(njobs, chunks);
}

size_t zn_decompress_temp_bytes(int64_t n, int k, int64_t chunk_bytes) {
  return zn_decompress_batch_temp_bytes(1, &n, k, &chunk_bytes);
}

int zn_decompress_batch(int njobs, const void* const* blobs, const int64_t* blob_bytes, const int64_t* n, int k,
                        int reorder, const int* ndim, const int64_t* chunk_bytes, const int64_t* n_comp,
                        void* const* out, int32_t* status, void* temp, size_t temp_bytes, void* stream) {
  if (njobs < 0 || (k != 1 && k != 2 && k != 4 && k != 8) || (reorder && k != 2 && k != 4))
    return set_error(ZN_ERR_INVALID, "zn_decompress: bad arguments");
  if (njobs == 0) return ZN_OK;
  NvtxScope range("zn_decompress_batch");
  if (!temp || temp_bytes < zn_decompress_batch_temp_bytes(njobs, n, k, chunk_bytes))
    return set_error(ZN_ERR_SPACE, "zn_decompress: temp buffer too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* tb = static_cast<uint8_t*>(temp);
  int64_t total_chunks = 0;
  for (int i = 0; i < njobs; ++i) total_chunks += n[i] > 0 && chunk_bytes[i] > 0 ? cdiv(n[i], chunk_bytes[i]) : 0;
  uint8_t* region = tb + job_table_bytes<DecArgs>(njobs, total_chunks);
  std::vector<DecArgs> jobs;
  jobs.reserve(static_cast<size_t>(njobs));
  int64_t chunk0 = 0;
  for (int i = 0; i < njobs; ++i) {
    if (n[i] < 0 || chunk_bytes[i] <= 0 || ndim[i] < 0 || ndim[i] > 64 || n_comp[i] < -1 ||
        (reinterpret_cast<uintptr_t>(blobs[i]) & 7))
      return set_error(ZN_ERR_INVALID, "zn_decompress: bad arguments (job %d)", i);
    if (n[i] == 0) continue;
    DecArgs a{};
    a.blob = static_cast<const uint8_t*>(blobs[i]);
    a.blob_bytes = blob_bytes[i];
    a.n = n[i];
    a.C = chunk_bytes[i];
    a.nch = cdiv(n[i], chunk_bytes[i]);
    a.units = int64_t(k) * a.nch;
    if (a.nch > 0x7FFFFFFF || n_comp[i] > a.units) return set_error(ZN_ERR_INVALID, "zn_decompress: bad tables (job %d)", i);
    a.sizes_off = 24 + 8 * int64_t(ndim[i]);
    a.idx_off = a.sizes_off + 4 * a.units;
    a.n_comp = n_comp[i];  // -1: dscan_kernel reads it from the blob
    a.data_off = n_comp[i] < 0 ? -1 : align8(a.idx_off + 4 * a.n_comp);
    if (n_comp[i] >= 0 && a.blob_bytes < a.data_off)
      return set_error(ZN_ERR_INVALID, "zn_decompress: blob is truncated (job %d)", i);
    a.chunk0 = chunk0;
    a.out = static_cast<uint8_t*>(out[i]);
    a.status = status + i;
    a.src = reinterpret_cast<int64_t*>(region);
    a.overflow = region + size_t(a.units) * 8;
    region += dec_job_bytes(n[i], k, chunk_bytes[i]);
    chunk0 += a.nch;
    jobs.push_back(a);
  }
  const int nj = int(jobs.size());
  if (nj == 0) return ZN_OK;
  if (chunk0 > 0x7FFFFFFF) return set_error(ZN_ERR_INVALID, "zn_decompress: too many chunks");
  DecArgs* dj = reinterpret_cast<DecArgs*>(tb);
  // A single job goes to the scan kernel by value (it stores the table itself).
  FirstJob<DecArgs> fj{};
  if (nj == 1) {
    fj.job = jobs[0];
    fj.valid = 1;
  } else if (int rc = upload_jobs(jobs.data(), nj, dj, chunk0, s)) {
    return rc;
  }
  {
    TimedLaunch tl("dscan", s);
    dscan_kernel<<<unsigned(nj), kScanThreads, 0, s>>>(dj, fj, dj);
  }
  count_launch();
  if (int rc = check_launch("dscan_kernel")) return rc;
  switch (k * 2 + (reorder ? 1 : 0)) {
    case 2: return launch_decode<1, false>(dj, nj, chunk0, s);
    case 4: return launch_decode<2, false>(dj, nj, chunk0, s);
    case 5: return launch_decode<2, true>(dj, nj, chunk0, s);
    case 8: return launch_decode<4, false>(dj, nj, chunk0, s);
    case 9: return launch_decode<4, true>(dj, nj, chunk0, s);
    default: return launch_decode<8, false>(dj, nj, chunk0, s);
  }
}

int zn_decompress(const void* blob, int64_t blob_bytes, int64_t n, int k, int reorder, int ndim, int64_t chunk_bytes,
                  int64_t n_comp, void* out, int32_t* status, void* temp, size_t temp_bytes, void* stream) {
  return zn_decompress_batch(1, &blob, &blob_bytes, &n, k, reorder, &ndim, &chunk_bytes, &n_comp, &out, status, temp,
                             temp_bytes, stream);
}

}  // extern "C"
