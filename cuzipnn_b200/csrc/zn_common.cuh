// Shared definitions of the cuZipNN-B200 CUDA library (sm_100a).
//
// The codec splits each K-byte element into K byte planes (after the exponent bit reorder that
// the reference applies to bfloat16 and float32, src/cuzipnn/_kernels.py:17-31) and entropy-codes
// every (plane, chunk) unit with the ZNR2 interleaved-rANS payload format:
//   scale 12 bits (M = 4096), u32 states in [2^15, 2^31), 16-bit word I/O, sub-chunks of
//   roundup(ceil(m / n_sub), 128) symbols, each coded by 8 interleaved states with one word
//   stream each; round r / step i / lane l covers symbol r*128 + l*16 + i of the sub-chunk.
// The normative CPU statement of the format is oracle/zn_oracle.c; these kernels must produce
// byte-identical payloads and blobs.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/cuzipnn_b200.h"

namespace zn {

constexpr uint32_t kScaleBits = 12;
constexpr uint32_t kM = 1u << kScaleBits;
constexpr uint32_t kL = 1u << 15;  // rANS states live in [kL, 2^31)
constexpr int kLanes = 8;        // states per sub-chunk
constexpr int kSteps = 16;       // symbols per lane per round
constexpr int kRound = kLanes * kSteps;
constexpr int kMinSubLog2 = 2;   // n_sub in [4, 64] (src/cuzipnn/_nvcomp.py:16-17)
constexpr int kMaxSubLog2 = 6;
constexpr int64_t kMaxChunkBytes = 1 << 24;  // src/cuzipnn/_nvcomp.py:13

// Device-side error bits (OR-ed into a status word; never a trap).
constexpr int32_t kErrPayload = 1;   // malformed rANS payload
constexpr int32_t kErrStream = 2;    // word stream over- or under-run, bad final state
constexpr int32_t kErrTable = 4;     // stored-size / index tables inconsistent with the blob
constexpr int32_t kErrGeometry = 8;  // compressed planes of one chunk disagree on n_sub

__host__ __device__ inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }
__host__ __device__ inline int64_t align8(int64_t x) { return (x + 7) & ~int64_t(7); }

// Sub-chunk geometry of a unit of m symbols coded with 2^t sub-chunks.
struct Geom {
  int64_t sc;   // symbols per sub-chunk (multiple of kRound)
  int nu;       // non-empty sub-chunks
  int lw;       // bytes per stream-length field (one field per state)
};

__host__ __device__ inline Geom geom_of(int64_t m, int t) {
  Geom g;
  g.sc = cdiv(cdiv(m, int64_t(1) << t), kRound) * kRound;
  g.nu = int(cdiv(m, g.sc));
  g.lw = g.sc / kLanes < 65536 ? 2 : 4;  // a state emits at most one word per symbol
  return g;
}

// Payload layout: [t, 0, bitmap(32), 12-bit freqs, pad4] [8 * nu lengths, pad4] [8 * nu states]
// [8 * nu streams], the per-state fields in (sub-chunk, lane) order.
__host__ __device__ inline int64_t table_bytes(int np) { return (2 + 32 + (12 * np + 7) / 8 + 3) & ~int64_t(3); }
__host__ __device__ inline int64_t lengths_bytes(const Geom& g) { return (int64_t(g.nu) * kLanes * g.lw + 3) & ~int64_t(3); }
__host__ __device__ inline int64_t meta_bytes(int np, const Geom& g) {
  return table_bytes(np) + lengths_bytes(g) + int64_t(g.nu) * kLanes * 4;
}
// Meta bytes of any unit coded with 2^t sub-chunks (at most 8 * 2^t streams, 4-byte lengths).
__host__ __device__ inline int64_t max_meta_bytes(int t) {
  return table_bytes(256) + (int64_t(kLanes) * 4 << t) + (int64_t(kLanes) * 4 << t);
}
// Payload bound for any unit of at most m symbols: at most one word per symbol.
__host__ __device__ inline int64_t max_payload(int64_t m, int t) { return max_meta_bytes(t) + 2 * m; }

// Exponent bit reorder of src/cuzipnn/_kernels.py:17-31, on two bfloat16 packed in a u32 or on
// one float32: `s eeeeeeee m` -> `eeeeeeee s m`, and back.
__device__ __forceinline__ uint32_t reorder_bf16x2(uint32_t w) {
  return ((w << 1) & 0xFF00FF00u) | ((w >> 8) & 0x00800080u) | (w & 0x007F007Fu);
}
__device__ __forceinline__ uint32_t revert_bf16x2(uint32_t w) {
  return ((w >> 1) & 0x7F807F80u) | ((w << 8) & 0x80008000u) | (w & 0x007F007Fu);
}
__device__ __forceinline__ uint32_t reorder_f32(uint32_t w) {
  return ((w << 1) & 0xFF000000u) | ((w >> 8) & 0x00800000u) | (w & 0x007FFFFFu);
}
__device__ __forceinline__ uint32_t revert_f32(uint32_t w) {
  return ((w >> 1) & 0x7F800000u) | ((w << 8) & 0x80000000u) | (w & 0x007FFFFFu);
}

// Reorder (or revert) every element held in `n` consecutive u32 words of K-byte elements.
template <int K, bool REORDER, bool FORWARD>
__device__ __forceinline__ void reorder_words(uint32_t* w, int n) {
  if constexpr (REORDER) {
#pragma unroll
    for (int i = 0; i < n; ++i) {
      if constexpr (K == 2) w[i] = FORWARD ? reorder_bf16x2(w[i]) : revert_bf16x2(w[i]);
      else w[i] = FORWARD ? reorder_f32(w[i]) : revert_f32(w[i]);
    }
  }
}

__device__ __forceinline__ uint32_t get_byte(const uint32_t* w, int i) { return (w[i >> 2] >> (8 * (i & 3))) & 0xFF; }

// Plane-major byte transposes of 16 elements (16 * K bytes in `e`, little-endian) into K plane
// vectors of 16 bytes (`p[b][0..3]`) and back.  PRMT selects bytes from two registers.
template <int K>
__device__ __forceinline__ void elements_to_planes(const uint32_t* e, uint32_t (*p)[4]) {
  if constexpr (K == 1) {
#pragma unroll
    for (int i = 0; i < 4; ++i) p[0][i] = e[i];
  } else if constexpr (K == 2) {
    // e holds 8 words of 2 elements; plane 0 = low bytes, plane 1 = high bytes.
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      p[0][i] = __byte_perm(e[2 * i], e[2 * i + 1], 0x6420);
      p[1][i] = __byte_perm(e[2 * i], e[2 * i + 1], 0x7531);
    }
  } else if constexpr (K == 4) {
    // 16 words, one element each; plane b gathers byte b of 4 consecutive elements.
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t a = __byte_perm(e[4 * i], e[4 * i + 1], 0x5140);      // b0e0 b0e1 b1e0 b1e1
      uint32_t b = __byte_perm(e[4 * i + 2], e[4 * i + 3], 0x5140);  // b0e2 b0e3 b1e2 b1e3
      uint32_t c = __byte_perm(e[4 * i], e[4 * i + 1], 0x7362);      // b2e0 b2e1 b3e0 b3e1
      uint32_t d = __byte_perm(e[4 * i + 2], e[4 * i + 3], 0x7362);
      p[0][i] = __byte_perm(a, b, 0x5410);
      p[1][i] = __byte_perm(a, b, 0x7632);
      p[2][i] = __byte_perm(c, d, 0x5410);
      p[3][i] = __byte_perm(c, d, 0x7632);
    }
  } else {
    static_assert(K == 8, "element size");
#pragma unroll
    for (int b = 0; b < 8; ++b)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint32_t v = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int el = 4 * i + q;
          v |= ((e[2 * el + (b >> 2)] >> (8 * (b & 3))) & 0xFF) << (8 * q);
        }
        p[b][i] = v;
      }
  }
}

template <int K>
__device__ __forceinline__ void planes_to_elements(const uint32_t (*p)[4], uint32_t* e) {
  if constexpr (K == 1) {
#pragma unroll
    for (int i = 0; i < 4; ++i) e[i] = p[0][i];
  } else if constexpr (K == 2) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      e[2 * i] = __byte_perm(p[0][i], p[1][i], 0x5140);
      e[2 * i + 1] = __byte_perm(p[0][i], p[1][i], 0x7362);
    }
  } else if constexpr (K == 4) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t lo01 = __byte_perm(p[0][i], p[1][i], 0x5140);  // p0e0 p1e0 p0e1 p1e1
      uint32_t lo23 = __byte_perm(p[0][i], p[1][i], 0x7362);  // p0e2 p1e2 p0e3 p1e3
      uint32_t hi01 = __byte_perm(p[2][i], p[3][i], 0x5140);
      uint32_t hi23 = __byte_perm(p[2][i], p[3][i], 0x7362);
      e[4 * i] = __byte_perm(lo01, hi01, 0x5410);
      e[4 * i + 1] = __byte_perm(lo01, hi01, 0x7632);
      e[4 * i + 2] = __byte_perm(lo23, hi23, 0x5410);
      e[4 * i + 3] = __byte_perm(lo23, hi23, 0x7632);
    }
  } else {
    static_assert(K == 8, "element size");
#pragma unroll
    for (int w = 0; w < 32; ++w) {
      const int el = w >> 1, half = w & 1;
      uint32_t v = 0;
#pragma unroll
      for (int q = 0; q < 4; ++q) v |= ((p[4 * half + q][el >> 2] >> (8 * (el & 3))) & 0xFF) << (8 * q);
      e[w] = v;
    }
  }
}

// Loads and stores of 16-byte-element groups; `vec16` picks 16- or 8-byte transactions.
// nwords is a compile-time constant at every call: the loops unroll fully, so w stays in registers.
__device__ __forceinline__ void load_words(const uint8_t* p, uint32_t* w, int nwords, bool vec16) {
  if (vec16) {
#pragma unroll
    for (int i = 0; i < nwords; i += 4) {
      uint4 v = *reinterpret_cast<const uint4*>(p + 4 * i);
      w[i] = v.x; w[i + 1] = v.y; w[i + 2] = v.z; w[i + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < nwords; i += 2) {
      uint2 v = *reinterpret_cast<const uint2*>(p + 4 * i);
      w[i] = v.x; w[i + 1] = v.y;
    }
  }
}

__device__ __forceinline__ void store_words(uint8_t* p, const uint32_t* w, int nwords, bool vec16) {
  if (vec16) {
#pragma unroll
    for (int i = 0; i < nwords; i += 4) *reinterpret_cast<uint4*>(p + 4 * i) = make_uint4(w[i], w[i + 1], w[i + 2], w[i + 3]);
  } else {
#pragma unroll
    for (int i = 0; i < nwords; i += 2) *reinterpret_cast<uint2*>(p + 4 * i) = make_uint2(w[i], w[i + 1]);
  }
}

// A batch's job table in device memory: njobs structs, then (for more than one job) a map from
// global chunk index to job index, so that a CTA finds its job with one load instead of a binary
// search through the job structs (a chain of dependent loads at the start of every CTA).
template <class J>
__host__ __device__ constexpr size_t job_structs_bytes(int njobs) {
  return (size_t(njobs) * sizeof(J) + 255) & ~size_t(255);
}
template <class J>
__host__ __device__ constexpr size_t job_table_bytes(int njobs, int64_t total_chunks) {
  return job_structs_bytes<J>(njobs) + (njobs > 1 ? (size_t(total_chunks) * 4 + 255) & ~size_t(255) : 0);
}

// Index of the job whose chunk range holds global chunk `gchunk`.
template <class J>
__device__ __forceinline__ int find_job(const J* __restrict__ jobs, int njobs, int64_t gchunk) {
  if (njobs == 1) return 0;
  const int32_t* map = reinterpret_cast<const int32_t*>(reinterpret_cast<const uint8_t*>(jobs) + job_structs_bytes<J>(njobs));
  return __ldg(map + gchunk);
}

// Job tables reach device memory as kernel parameters (copied by the launch itself), so no host
// staging buffer is needed: each launch carries up to ~30 KB of jobs.  CTA q copies job q, and for
// a call of more than one job also writes the chunk -> job map over its job's chunk range
// [chunk0_q, chunk0_{q+1}) (behind the whole job table: job_table_bytes).
template <class T, int N>
struct UploadBatch {
  T items[N];
  int count;          // jobs in this launch
  int first;          // index of items[0] in the call's job table
  int njobs;          // jobs in the call
  int64_t end_chunk;  // first chunk after the launch's last job
};

template <class T, int N>
__global__ void upload_kernel(const __grid_constant__ UploadBatch<T, N> b, T* table) {
  static_assert(sizeof(T) % 4 == 0, "job size");
  const int q = blockIdx.x;
  const uint32_t* src = reinterpret_cast<const uint32_t*>(&b.items[q]);
  uint32_t* d = reinterpret_cast<uint32_t*>(table + b.first + q);
  for (int i = threadIdx.x; i < int(sizeof(T) / 4); i += blockDim.x) d[i] = src[i];
  if (b.njobs > 1) {
    int32_t* map = reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(table) + job_structs_bytes<T>(b.njobs));
    const int64_t c0 = b.items[q].chunk0, c1 = q + 1 < b.count ? b.items[q + 1].chunk0 : b.end_chunk;
    for (int64_t c = c0 + threadIdx.x; c < c1; c += blockDim.x) map[c] = b.first + q;
  }
}

// The one job of a single-job call, passed by value to the call's first kernel, which stores it
// into the job table for the kernels after it: such a call needs no upload launch.  valid = 0 when
// the table was uploaded.
template <class T>
struct FirstJob {
  T job;
  int valid;
};

// Store a job into its table slot, with the threads of one CTA.
template <class T>
__device__ __forceinline__ void store_job(const T& job, T* slot) {
  const uint32_t* s = reinterpret_cast<const uint32_t*>(&job);
  uint32_t* d = reinterpret_cast<uint32_t*>(slot);
  for (int i = threadIdx.x; i < int(sizeof(T) / 4); i += blockDim.x) d[i] = s[i];
}

// ---- host side ------------------------------------------------------------------------------

// Records the error of the last failing call of this thread and returns its status.
int set_error(int status, const char* fmt, ...);
int check_launch(const char* what);
void count_launch(int n = 1);
int set_max_smem(const void* func, int bytes);

// Copy `count` host structs to device memory at dev, on stream s, through kernel parameters, with
// the chunk -> job map behind them for more than one job (job_table_bytes): one launch per ~30 KB
// of jobs.
template <class T, int N>
int upload_batches(const T* host, int count, T* dev, int64_t total_chunks, cudaStream_t s) {
  for (int i = 0; i < count; i += N) {
    UploadBatch<T, N> b;
    b.count = count - i < N ? count - i : N;
    b.first = i;
    b.njobs = count;
    b.end_chunk = i + b.count < count ? host[i + b.count].chunk0 : total_chunks;
    for (int q = 0; q < b.count; ++q) b.items[q] = host[i + q];
    upload_kernel<T, N><<<unsigned(b.count), 256, 0, s>>>(b, dev);
    count_launch();
    if (int rc = check_launch("upload_kernel")) return rc;
  }
  return ZN_OK;
}

template <class T>
int upload_jobs(const T* host, int count, T* dev, int64_t total_chunks, cudaStream_t s) {
  // A call with a few jobs (one tensor) takes a small parameter block, since the launch cost
  // grows with the block's size.
  constexpr int N = 30000 / int(sizeof(T)) > 0 ? 30000 / int(sizeof(T)) : 1;
  return count <= 4 ? upload_batches<T, 4>(host, count, dev, total_chunks, s)
                    : upload_batches<T, N>(host, count, dev, total_chunks, s);
}

// An NVTX range over a scope of host code (entry points), visible to Nsight tools.
struct NvtxScope {
  explicit NvtxScope(const char* name);
  ~NvtxScope();
};

// Opt-in event timing of one kernel kind (zn_timing_enable): bracket a launch with
// TimedLaunch t("decode", stream); ... launch ...; (the destructor records the end event).  It
// also opens an NVTX range named after the kernel kind for the launch.
struct TimedLaunch {
  TimedLaunch(const char* kernel, cudaStream_t stream);
  ~TimedLaunch();
  int slot;
  cudaStream_t stream;
};

}  // namespace zn
