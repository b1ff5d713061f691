// Byte-plane seam kernels: the drop-in replacements of the reference's Triton kernels
// (src/cuzipnn/_kernels.py:34-188).  The whole-tensor codec does not use them (its split and
// merge are fused into the entropy coder and the packer); they serve callers of the seam API.
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
template <int K>
__global__ void split_kernel(const typename Word<K>::T* __restrict__ x, int64_t n, bool reorder,
                             uint8_t* __restrict__ planar, int64_t stride) {
  for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < n; e += int64_t(gridDim.x) * blockDim.x) {
    uint64_t u = x[e];
    if constexpr (K == 2 || K == 4) {
      if (reorder) u = reorder_elem<K>(u, true);
    }
#pragma unroll
    for (int b = 0; b < K; ++b) planar[b * stride + e] = uint8_t(u >> (8 * b));
  }
}

// src/cuzipnn/_kernels.py:57-105: stream b of chunk j is at base + src_tbl[b * nch + j].
template <int K>
__global__ void merge_kernel(const int64_t* __restrict__ src_tbl, const uint8_t* __restrict__ base,
                             typename Word<K>::T* __restrict__ out, int64_t n, int64_t chunk, int64_t nch,
                             bool reorder) {
  for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < n; e += int64_t(gridDim.x) * blockDim.x) {
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

extern "C" {

int zn_split(const void* x, int64_t n, int k, int reorder, void* planar, int64_t stride, void* stream) {
  if (n < 0 || stride < n || (k != 1 && k != 2 && k != 4 && k != 8) || (reorder && k != 2 && k != 4))
    return set_error(ZN_ERR_INVALID, "zn_split: bad arguments (n=%lld k=%d stride=%lld)", (long long)n, k,
                     (long long)stride);
  if (n == 0) return ZN_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int threads = 256, grid = grid_for(n, threads);
  uint8_t* p = static_cast<uint8_t*>(planar);
  switch (k) {
    case 1: split_kernel<1><<<grid, threads, 0, s>>>(static_cast<const uint8_t*>(x), n, false, p, stride); break;
    case 2: split_kernel<2><<<grid, threads, 0, s>>>(static_cast<const uint16_t*>(x), n, reorder, p, stride); break;
    case 4: split_kernel<4><<<grid, threads, 0, s>>>(static_cast<const uint32_t*>(x), n, reorder, p, stride); break;
    default: split_kernel<8><<<grid, threads, 0, s>>>(static_cast<const unsigned long long*>(x), n, false, p, stride); break;
  }
  count_launch();
  return check_launch("zn_split");
}

int zn_merge(const int64_t* src_tbl, const void* base, void* out, int64_t n, int k, int64_t chunk_bytes,
             int reorder, void* stream) {
  if (n < 0 || chunk_bytes <= 0 || (k != 1 && k != 2 && k != 4 && k != 8) || (reorder && k != 2 && k != 4))
    return set_error(ZN_ERR_INVALID, "zn_merge: bad arguments");
  if (n == 0) return ZN_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t nch = cdiv(n, chunk_bytes);
  const int threads = 256, grid = grid_for(n, threads);
  const uint8_t* b = static_cast<const uint8_t*>(base);
  switch (k) {
    case 1: merge_kernel<1><<<grid, threads, 0, s>>>(src_tbl, b, static_cast<uint8_t*>(out), n, chunk_bytes, nch, false); break;
    case 2: merge_kernel<2><<<grid, threads, 0, s>>>(src_tbl, b, static_cast<uint16_t*>(out), n, chunk_bytes, nch, reorder); break;
    case 4: merge_kernel<4><<<grid, threads, 0, s>>>(src_tbl, b, static_cast<uint32_t*>(out), n, chunk_bytes, nch, reorder); break;
    default: merge_kernel<8><<<grid, threads, 0, s>>>(src_tbl, b, static_cast<unsigned long long*>(out), n, chunk_bytes, nch, false); break;
  }
  count_launch();
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
