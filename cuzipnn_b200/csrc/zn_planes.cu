// Byte-plane seam kernels: the drop-in replacements of the reference's Triton kernels
// (src/cuzipnn/_kernels.py:34-188).  The whole-tensor codec does not use them (its split and
// merge are fused into the entropy coder and the packer); they serve callers of the seam API.
//
// split and merge move 16 elements per thread and step: coalesced 16-byte loads of the elements
// (or of each plane's 16 bytes), the byte transpose in registers (byte permutes), and 16-byte
// stores per plane (8-byte or byte stores when a plane's start is not so aligned).  Elements
// after the last whole group of 16, and pointers that are not 8-byte aligned, take the scalar
// kernels.
#include "zn_common.cuh"

namespace zn {
namespace {

template <int K>
struct Word;
template <> struct Word<1> { using T = uint8_t; };
template <> struct Word<2> { using T = uint16_t; };
template <> struct Word<4> { using T = uint32_t; };
template <> struct Word<8> { using T = unsigned long long; };

template <int K>
__device__ __forceinline__ uint64_t reorder_elem(uint64_t u, bool forward) {
  constexpr int W = 8 * K;
  if (forward) {
    uint64_t exp = (u >> (W - 9)) & 0xFF, sign = u >> (W - 1), mant = u & ((uint64_t(1) << (W - 9)) - 1);
    return (exp << (W - 8)) | (sign << (W - 9)) | mant;
  }
  uint64_t exp = u >> (W - 8), sign = (u >> (W - 9)) & 1, mant = u & ((uint64_t(1) << (W - 9)) - 1);
  return (sign << (W - 1)) | (exp << (W - 9)) | mant;
}

// src/cuzipnn/_kernels.py:34-54: byte b of element e goes to planar[b * stride + e].
// Elements e0 .. n - 1 (all of them, or the tail after the 16-element groups).
template <int K>
__global__ void split_kernel(const typename Word<K>::T* __restrict__ x, int64_t e0, int64_t n, bool reorder,
                             uint8_t* __restrict__ planar, int64_t stride) {
  for (int64_t e = e0 + int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < n; e += int64_t(gridDim.x) * blockDim.x) {
    uint64_t u = x[e];
    if constexpr (K == 2 || K == 4) {
      if (reorder) u = reorder_elem<K>(u, true);
    }
#pragma unroll
    for (int b = 0; b < K; ++b) planar[b * stride + e] = uint8_t(u >> (8 * b));
  }
}

// Split 16 elements per thread and step (groups g of elements 16 g .. 16 g + 15).  x16: x is
// 16-byte aligned (else 8); st: 2 = each plane's group start is 16-byte aligned (planar and
// stride), 1 = 8-byte aligned, 0 = byte stores.
template <int K, bool REORDER>
__global__ void __launch_bounds__(256) split16_kernel(const uint8_t* __restrict__ x, int64_t groups, bool x16,
                                                      uint8_t* __restrict__ planar, int64_t stride, int st) {
  for (int64_t g = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; g < groups; g += int64_t(gridDim.x) * blockDim.x) {
    uint32_t e[4 * K];
    load_words(x + g * 16 * K, e, 4 * K, x16);
    reorder_words<K, REORDER, true>(e, 4 * K);
    uint32_t p[K][4];
    elements_to_planes<K>(e, p);
#pragma unroll
    for (int b = 0; b < K; ++b) {
      uint8_t* d = planar + b * stride + g * 16;
      if (st == 2) {
        *reinterpret_cast<uint4*>(d) = make_uint4(p[b][0], p[b][1], p[b][2], p[b][3]);
      } else if (st == 1) {
        reinterpret_cast<uint2*>(d)[0] = make_uint2(p[b][0], p[b][1]);
        reinterpret_cast<uint2*>(d)[1] = make_uint2(p[b][2], p[b][3]);
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) d[i] = uint8_t(p[b][i >> 2] >> (8 * (i & 3)));
      }
    }
  }
}

// Merge 16 elements per thread and step.  A group inside one chunk reads each plane's 16 bytes
// with two 8-byte loads (byte loads if that source is not 8-byte aligned); a group that straddles
// a chunk boundary gathers byte by byte.  out16: out is 16-byte aligned (else 8).
template <int K, bool REORDER>
__global__ void __launch_bounds__(256) merge16_kernel(const int64_t* __restrict__ src_tbl,
                                                      const uint8_t* __restrict__ base, uint8_t* __restrict__ out,
                                                      int64_t groups, int64_t chunk, int64_t nch, bool out16) {
  for (int64_t g = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; g < groups; g += int64_t(gridDim.x) * blockDim.x) {
    const int64_t e0 = g * 16, j = e0 / chunk, o = e0 - j * chunk;
    uint32_t p[K][4];
    if (o + 16 <= chunk) {
#pragma unroll
      for (int b = 0; b < K; ++b) {
        const uint8_t* sp = base + __ldg(src_tbl + b * nch + j) + o;
        if ((reinterpret_cast<uintptr_t>(sp) & 7) == 0) {
          const uint2 v0 = reinterpret_cast<const uint2*>(sp)[0], v1 = reinterpret_cast<const uint2*>(sp)[1];
          p[b][0] = v0.x; p[b][1] = v0.y; p[b][2] = v1.x; p[b][3] = v1.y;
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i) p[b][i] = 0;
#pragma unroll
          for (int i = 0; i < 16; ++i) p[b][i >> 2] |= uint32_t(sp[i]) << (8 * (i & 3));
        }
      }
    } else {
#pragma unroll
      for (int b = 0; b < K; ++b)
#pragma unroll
        for (int i = 0; i < 4; ++i) p[b][i] = 0;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int64_t e = e0 + i, jj = e / chunk, oo = e - jj * chunk;
#pragma unroll
        for (int b = 0; b < K; ++b) p[b][i >> 2] |= uint32_t(base[src_tbl[b * nch + jj] + oo]) << (8 * (i & 3));
      }
    }
    uint32_t e[4 * K];
    planes_to_elements<K>(p, e);
    reorder_words<K, REORDER, false>(e, 4 * K);
    store_words(out + e0 * K, e, 4 * K, out16);
  }
}

// src/cuzipnn/_kernels.py:57-105: stream b of chunk j is at base + src_tbl[b * nch + j].
// Elements e0 .. n - 1 (all of them, or the tail after the 16-element groups).
template <int K>
__global__ void merge_kernel(const int64_t* __restrict__ src_tbl, const uint8_t* __restrict__ base,
                             typename Word<K>::T* __restrict__ out, int64_t e0, int64_t n, int64_t chunk, int64_t nch,
                             bool reorder) {
  for (int64_t e = e0 + int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < n; e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t j = e / chunk, o = e - j * chunk;
    uint64_t u = 0;
#pragma unroll
    for (int b = 0; b < K; ++b) u |= uint64_t(base[src_tbl[b * nch + j] + o]) << (8 * b);
    if constexpr (K == 2 || K == 4) {
      if (reorder) u = reorder_elem<K>(u, false);
    }
    out[e] = typename Word<K>::T(u);
  }
}

// src/cuzipnn/_kernels.py:108-131: chunk i (blockIdx.x), tile blockIdx.y of 8 KiB.
constexpr int kCopyTile = 8192;

__global__ void copy_chunks_kernel(const int64_t* __restrict__ src_tbl, const int64_t* __restrict__ dst_tbl,
                                   const int64_t* __restrict__ nbytes, bool pad) {
  const int64_t i = blockIdx.x;
  const int64_t nb = nbytes[i];
  const int64_t t0 = int64_t(blockIdx.y) * kCopyTile;
  if (nb <= 0 || t0 >= nb) return;
  const uint8_t* src = reinterpret_cast<const uint8_t*>(src_tbl[i]);
  uint8_t* dst = reinterpret_cast<uint8_t*>(dst_tbl[i]);
  const int64_t end = min(nb, t0 + kCopyTile);
  const int64_t wend = t0 + ((end - t0) & ~int64_t(7));
  for (int64_t o = t0 + 8 * threadIdx.x; o < wend; o += 8 * blockDim.x)
    *reinterpret_cast<uint64_t*>(dst + o) = *reinterpret_cast<const uint64_t*>(src + o);
  if (threadIdx.x < 8) {
    const int64_t o = wend + threadIdx.x;
    if (o < end) dst[o] = src[o];
    else if (pad && end == nb && o < align8(nb)) dst[o] = 0;
  }
}

}  // namespace
}  // namespace zn

using namespace zn;

static int grid_for(int64_t n, int threads) {
  int64_t g = cdiv(n, threads);
  return int(g < 148 * 64 ? (g < 1 ? 1 : g) : 148 * 64);
}

template <int K, bool R>
static void split16(const void* x, int64_t groups, bool x16, uint8_t* p, int64_t stride, int st, cudaStream_t s) {
  split16_kernel<K, R><<<grid_for(groups, 256), 256, 0, s>>>(static_cast<const uint8_t*>(x), groups, x16, p, stride, st);
}

template <int K, bool R>
static void merge16(const int64_t* tbl, const uint8_t* b, void* out, int64_t groups, int64_t chunk, int64_t nch,
                    bool out16, cudaStream_t s) {
  merge16_kernel<K, R><<<grid_for(groups, 256), 256, 0, s>>>(tbl, b, static_cast<uint8_t*>(out), groups, chunk, nch,
                                                             out16);
}

extern "C" {

int zn_split(const void* x, int64_t n, int k, int reorder, void* planar, int64_t stride, void* stream) {
  if (n < 0 || stride < n || (k != 1 && k != 2 && k != 4 && k != 8) || (reorder && k != 2 && k != 4))
    return set_error(ZN_ERR_INVALID, "zn_split: bad arguments (n=%lld k=%d stride=%lld)", (long long)n, k,
                     (long long)stride);
  if (n == 0) return ZN_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* p = static_cast<uint8_t*>(planar);
  const uintptr_t xa = reinterpret_cast<uintptr_t>(x);
  // Groups of 16 elements from an 8-byte aligned x; the rest element by element.
  const int64_t groups = (xa & 7) == 0 ? n / 16 : 0;
  int launches = 0;
  if (groups > 0) {
    const bool x16 = (xa & 15) == 0;
    const uint64_t pa = uint64_t(reinterpret_cast<uintptr_t>(p)) | uint64_t(stride);
    const int st = (pa & 15) == 0 ? 2 : (pa & 7) == 0 ? 1 : 0;
    switch (k * 2 + (reorder ? 1 : 0)) {
      case 2: split16<1, false>(x, groups, x16, p, stride, st, s); break;
      case 4: split16<2, false>(x, groups, x16, p, stride, st, s); break;
      case 5: split16<2, true>(x, groups, x16, p, stride, st, s); break;
      case 8: split16<4, false>(x, groups, x16, p, stride, st, s); break;
      case 9: split16<4, true>(x, groups, x16, p, stride, st, s); break;
      default: split16<8, false>(x, groups, x16, p, stride, st, s); break;
    }
    ++launches;
  }
  const int64_t e0 = groups * 16;
  if (e0 < n) {
    const int threads = 256, grid = grid_for(n - e0, threads);
    switch (k) {
      case 1: split_kernel<1><<<grid, threads, 0, s>>>(static_cast<const uint8_t*>(x), e0, n, false, p, stride); break;
      case 2: split_kernel<2><<<grid, threads, 0, s>>>(static_cast<const uint16_t*>(x), e0, n, reorder, p, stride); break;
      case 4: split_kernel<4><<<grid, threads, 0, s>>>(static_cast<const uint32_t*>(x), e0, n, reorder, p, stride); break;
      default: split_kernel<8><<<grid, threads, 0, s>>>(static_cast<const unsigned long long*>(x), e0, n, false, p, stride); break;
    }
    ++launches;
  }
  count_launch(launches);
  return check_launch("zn_split");
}

int zn_merge(const int64_t* src_tbl, const void* base, void* out, int64_t n, int k, int64_t chunk_bytes,
             int reorder, void* stream) {
  if (n < 0 || chunk_bytes <= 0 || (k != 1 && k != 2 && k != 4 && k != 8) || (reorder && k != 2 && k != 4))
    return set_error(ZN_ERR_INVALID, "zn_merge: bad arguments");
  if (n == 0) return ZN_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t nch = cdiv(n, chunk_bytes);
  const uint8_t* b = static_cast<const uint8_t*>(base);
  const uintptr_t oa = reinterpret_cast<uintptr_t>(out);
  // Groups of 16 elements into an 8-byte aligned out; the rest element by element.
  const int64_t groups = (oa & 7) == 0 ? n / 16 : 0;
  int launches = 0;
  if (groups > 0) {
    const bool o16 = (oa & 15) == 0;
    switch (k * 2 + (reorder ? 1 : 0)) {
      case 2: merge16<1, false>(src_tbl, b, out, groups, chunk_bytes, nch, o16, s); break;
      case 4: merge16<2, false>(src_tbl, b, out, groups, chunk_bytes, nch, o16, s); break;
      case 5: merge16<2, true>(src_tbl, b, out, groups, chunk_bytes, nch, o16, s); break;
      case 8: merge16<4, false>(src_tbl, b, out, groups, chunk_bytes, nch, o16, s); break;
      case 9: merge16<4, true>(src_tbl, b, out, groups, chunk_bytes, nch, o16, s); break;
      default: merge16<8, false>(src_tbl, b, out, groups, chunk_bytes, nch, o16, s); break;
    }
    ++launches;
  }
  const int64_t e0 = groups * 16;
  if (e0 < n) {
    const int threads = 256, grid = grid_for(n - e0, threads);
    switch (k) {
      case 1: merge_kernel<1><<<grid, threads, 0, s>>>(src_tbl, b, static_cast<uint8_t*>(out), e0, n, chunk_bytes, nch, false); break;
      case 2: merge_kernel<2><<<grid, threads, 0, s>>>(src_tbl, b, static_cast<uint16_t*>(out), e0, n, chunk_bytes, nch, reorder); break;
      case 4: merge_kernel<4><<<grid, threads, 0, s>>>(src_tbl, b, static_cast<uint32_t*>(out), e0, n, chunk_bytes, nch, reorder); break;
      default: merge_kernel<8><<<grid, threads, 0, s>>>(src_tbl, b, static_cast<unsigned long long*>(out), e0, n, chunk_bytes, nch, false); break;
    }
    ++launches;
  }
  count_launch(launches);
  return check_launch("zn_merge");
}

int zn_copy_chunks(const int64_t* src_tbl, const int64_t* dst_tbl, const int64_t* nbytes, int64_t count,
                   int64_t max_bytes, int pad, void* stream) {
  if (count < 0 || max_bytes < 0 || count > 0x7FFFFFFF) return set_error(ZN_ERR_INVALID, "zn_copy_chunks: bad arguments");
  if (count == 0 || max_bytes == 0) return ZN_OK;
  const int64_t tiles = cdiv(max_bytes, kCopyTile);
  if (tiles > 65535) return set_error(ZN_ERR_INVALID, "zn_copy_chunks: max_bytes too large");
  copy_chunks_kernel<<<dim3(unsigned(count), unsigned(tiles)), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      src_tbl, dst_tbl, nbytes, pad != 0);
  count_launch();
  return check_launch("zn_copy_chunks");
}

}  // extern "C"
