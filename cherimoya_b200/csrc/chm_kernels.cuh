// chm_kernels.cuh -- device kernels of the Cherimoya B200 engine.
//
// Activation layout in HBM: the residual stream of a batch is one row-major
// matrix X[(n * L + l) * CP + c] (NLC, channels innermost, padded to CP, a
// multiple of 64; padded channels hold 0). act_t is float (fp32 mode) or
// __nv_bfloat16 (bf16 mode).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <type_traits>

#include "chm_ptx.cuh"

namespace chm {

constexpr int kStemTaps = 21;   // iconv kernel size (upstream cherimoya.py:173)
constexpr int kStemPad = 10;
constexpr int kHeadTaps = 75;   // fconv kernel size (upstream cherimoya.py:182-184)
constexpr int kHeadPad = 37;
constexpr int kTileRows = 128;  // MMA M

enum : int { kStatusOk = 0, kStatusTimeout = 5 };

template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// Loads / stores of `N` consecutive activations (N * sizeof(act_t) is 4, 8
// or 16 bytes and the address is aligned to it).
template <typename T, int N> struct Vec;
template <int N> struct Vec<float, N> {
  static __device__ __forceinline__ void load(const float* p, float (&v)[N]) {
    if constexpr (N == 8) {
      const float4 t = *reinterpret_cast<const float4*>(p);
      const float4 u = *reinterpret_cast<const float4*>(p + 4);
      v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
      v[4] = u.x; v[5] = u.y; v[6] = u.z; v[7] = u.w;
    } else if constexpr (N == 4) {
      float4 t = *reinterpret_cast<const float4*>(p);
      v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
    } else if constexpr (N == 2) {
      float2 t = *reinterpret_cast<const float2*>(p);
      v[0] = t.x; v[1] = t.y;
    } else {
#pragma unroll
      for (int i = 0; i < N; ++i) v[i] = p[i];
    }
  }
  static __device__ __forceinline__ void store(float* p, const float (&v)[N]) {
    if constexpr (N == 4) {
      *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    } else if constexpr (N == 2) {
      *reinterpret_cast<float2*>(p) = make_float2(v[0], v[1]);
    } else {
#pragma unroll
      for (int i = 0; i < N; ++i) p[i] = v[i];
    }
  }
};
template <int N> struct Vec<__nv_bfloat16, N> {
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float (&v)[N]) {
    if constexpr (N == 8) {
      const uint4 t = *reinterpret_cast<const uint4*>(p);
      v[0] = __uint_as_float(t.x << 16); v[1] = __uint_as_float(t.x & 0xFFFF0000u);
      v[2] = __uint_as_float(t.y << 16); v[3] = __uint_as_float(t.y & 0xFFFF0000u);
      v[4] = __uint_as_float(t.z << 16); v[5] = __uint_as_float(t.z & 0xFFFF0000u);
      v[6] = __uint_as_float(t.w << 16); v[7] = __uint_as_float(t.w & 0xFFFF0000u);
    } else if constexpr (N == 4) {
      uint2 t = *reinterpret_cast<const uint2*>(p);
      __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(&t.x);
      __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&t.y);
      float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
      v[0] = fa.x; v[1] = fa.y; v[2] = fb.x; v[3] = fb.y;
    } else if constexpr (N == 2) {
      __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(p);
      float2 fa = __bfloat1622float2(a);
      v[0] = fa.x; v[1] = fa.y;
    } else {
#pragma unroll
      for (int i = 0; i < N; ++i) v[i] = __bfloat162float(p[i]);
    }
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, const float (&v)[N]) {
    if constexpr (N == 4) {
      uint2 t = make_uint2(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]));
      *reinterpret_cast<uint2*>(p) = t;
    } else if constexpr (N == 2) {
      *reinterpret_cast<uint32_t*>(p) = pack_bf16x2(v[0], v[1]);
    } else {
#pragma unroll
      for (int i = 0; i < N; ++i) p[i] = __float2bfloat16_rn(v[i]);
    }
  }
};

__device__ __forceinline__ void unpack4(const uint2& t, float (&v)[4]) {
  v[0] = __uint_as_float(t.x << 16);
  v[1] = __uint_as_float(t.x & 0xFFFF0000u);
  v[2] = __uint_as_float(t.y << 16);
  v[3] = __uint_as_float(t.y & 0xFFFF0000u);
}
__device__ __forceinline__ void unpack4(const float4& t, float (&v)[4]) {
  v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
}

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 t = *reinterpret_cast<const uint4*>(p);
  v[0] = __uint_as_float(t.x << 16); v[1] = __uint_as_float(t.x & 0xFFFF0000u);
  v[2] = __uint_as_float(t.y << 16); v[3] = __uint_as_float(t.y & 0xFFFF0000u);
  v[4] = __uint_as_float(t.z << 16); v[5] = __uint_as_float(t.z & 0xFFFF0000u);
  v[6] = __uint_as_float(t.w << 16); v[7] = __uint_as_float(t.w & 0xFFFF0000u);
}
__device__ __forceinline__ void load8(const float* p, float (&v)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  const float4 b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

struct Raw8f {
  float4 a, b;
};
template <typename R, typename T>
__device__ __forceinline__ R ldraw(const T* p) {
  if constexpr (sizeof(R) == 16) {
    return *reinterpret_cast<const R*>(p);
  } else {
    R r;
    r.a = *reinterpret_cast<const float4*>(p);
    r.b = *reinterpret_cast<const float4*>(p + 4);
    return r;
  }
}
__device__ __forceinline__ void unpack8(const uint4& t, float (&v)[8]) {
  v[0] = __uint_as_float(t.x << 16); v[1] = __uint_as_float(t.x & 0xFFFF0000u);
  v[2] = __uint_as_float(t.y << 16); v[3] = __uint_as_float(t.y & 0xFFFF0000u);
  v[4] = __uint_as_float(t.z << 16); v[5] = __uint_as_float(t.z & 0xFFFF0000u);
  v[6] = __uint_as_float(t.w << 16); v[7] = __uint_as_float(t.w & 0xFFFF0000u);
}
__device__ __forceinline__ void unpack8(const Raw8f& t, float (&v)[8]) {
  v[0] = t.a.x; v[1] = t.a.y; v[2] = t.a.z; v[3] = t.a.w;
  v[4] = t.b.x; v[5] = t.b.y; v[6] = t.b.z; v[7] = t.b.w;
}

// 16 bytes of activations plus the matching fp32 MLP outputs (raw bits).
template <typename act_t>
__device__ __forceinline__ uint4 add_residual(const uint4& x, const uint32_t* d) {
  if constexpr (sizeof(act_t) == 2) {
    float v[8];
    unpack8(x, v);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] += __uint_as_float(d[e]);
    return make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                      pack_bf16x2(v[6], v[7]));
  } else {
    return make_uint4(__float_as_uint(__uint_as_float(x.x) + __uint_as_float(d[0])),
                      __float_as_uint(__uint_as_float(x.y) + __uint_as_float(d[1])),
                      __float_as_uint(__uint_as_float(x.z) + __uint_as_float(d[2])),
                      __float_as_uint(__uint_as_float(x.w) + __uint_as_float(d[3])));
  }
}

__host__ __device__ __forceinline__ int kHeadThreadsRows(int chunks) { return 128 / chunks; }

template <typename act_t>
__device__ __forceinline__ void unpack_chunk(const uint4& t, float (&v)[16 / sizeof(act_t)]) {
  if constexpr (sizeof(act_t) == 2) {
    unpack8(t, v);
  } else {
    v[0] = __uint_as_float(t.x); v[1] = __uint_as_float(t.y);
    v[2] = __uint_as_float(t.z); v[3] = __uint_as_float(t.w);
  }
}

// ============================================================== input
// Input of the stem, one of:
//  kInDense : x (B, 4, L) fp32 or bf16 (NCL), any values
//  kInBases : bases (B, L) int8, base b in 0..3 -> one-hot column, other
//             values -> all-zero column
//  kInIsm   : mutant m of an ISM pass: sequence seq = m_base / per_seq ... the
//             mutant's bases are its reference's with one substitution
enum : int { kInDense = 0, kInBases = 1, kInIsm = 2 };

struct StemInput {
  const void* x;          // kInDense
  int x_bf16;             // kInDense: element type
  const int8_t* bases;    // kInBases / kInIsm: (n_ref, L)
  long long mut0;         // kInIsm: global index of this pass's first mutant
  int ism_start;          // kInIsm: first mutated position
  int ism_width;          // kInIsm: number of mutated positions
};

// Value of input channel k (0..3) at position p (0 <= p < L) of batch row b.
template <int kIn>
__device__ __forceinline__ void stem_column(const StemInput& in, int L, int b, int p,
                                            float (&col)[4]) {
  if constexpr (kIn == kInDense) {
    if (in.x_bf16) {
      const __nv_bfloat16* x = static_cast<const __nv_bfloat16*>(in.x);
#pragma unroll
      for (int k = 0; k < 4; ++k) col[k] = __bfloat162float(x[((long long)b * 4 + k) * L + p]);
    } else {
      const float* x = static_cast<const float*>(in.x);
#pragma unroll
      for (int k = 0; k < 4; ++k) col[k] = x[((long long)b * 4 + k) * L + p];
    }
  } else {
    int base;
    if constexpr (kIn == kInBases) {
      base = in.bases[(long long)b * L + p];
    } else {
      // mutant index -> (reference n, position offset w, alternative k)
      const long long m = in.mut0 + b;
      const long long per_seq = 3LL * in.ism_width;
      const int n = static_cast<int>(m / per_seq);
      const int rem = static_cast<int>(m - (long long)n * per_seq);
      const int w = rem / 3, k = rem - 3 * (rem / 3);
      const int mp = in.ism_start + w;
      base = in.bases[(long long)n * L + p];
      if (p == mp) base = ((in.bases[(long long)n * L + mp] & 3) + 1 + k) & 3;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) col[k] = (base == k) ? 1.0f : 0.0f;
  }
}

// ============================================================== stem, tcgen05
// Stem as an im2col GEMM over 128-row tiles of the flattened (B*L) rows:
//   A[r, 4t + k] = x[b, k, l + t - 10]  (K = 84 tap-major, padded to 128)
//   X0[r, c] = gelu_tanh(bias[c] + sum_kk A[r, kk] W[c, kk])
// (upstream cherimoya.py:173-174, 373). W is packed as bf16 hi + lo (two
// MMAs carry it to ~16 bits); one-hot / base inputs are exact in bf16, a
// dense fp32 input is split into hi + lo as well (third MMA).
namespace sm {
constexpr int kK = 128;            // padded im2col width
constexpr int kThreads = 128;
}  // namespace sm

__host__ __device__ constexpr uint32_t stem_smem_bytes(int CP, int a_splits) {
  return static_cast<uint32_t>(2 * CP * sm::kK * 2 + a_splits * kTileRows * sm::kK * 2 + 64 +
                               1024);
}

template <typename act_t, int kIn, int kASplits>
__global__ void __launch_bounds__(sm::kThreads) stem_mma_kernel(StemInput in,
                                                                const uint8_t* __restrict__ wpk,
                                                                const float* __restrict__ bias,
                                                                act_t* X, long long rows, int L,
                                                                int C, int CP, int n_tiles,
                                                                int* status) {
  using namespace sm;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sB = smem;                                 // [hi | lo] CP x 128
  uint8_t* sA = sB + 2 * CP * kK * 2;                 // [kASplits] 128 x 128
  uint64_t* bar = reinterpret_cast<uint64_t*>(sA + kASplits * kTileRows * kK * 2);
  uint32_t* slot = reinterpret_cast<uint32_t*>(bar + 1);
  const int tid = threadIdx.x, warp = tid >> 5;
  if (warp == 0) tmem_alloc(slot, 256);
  if (tid == 0) {
    mbar_init(bar, 1);
    mbar_init_fence();
  }
  {
    const uint4* g = reinterpret_cast<const uint4*>(wpk);
    uint4* d = reinterpret_cast<uint4*>(sB);
    for (int i = tid; i < 2 * CP * kK * 2 / 16; i += blockDim.x) d[i] = g[i];
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *slot;
  const uint32_t sA_addr = smem_u32(sA), sB_addr = smem_u32(sB);
  const uint32_t idesc = idesc_bf16(kTileRows, CP);
  const uint32_t lane_sel = static_cast<uint32_t>(warp * 32) << 16;
  uint32_t it = 0;
  for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
    const long long r = (long long)tile * kTileRows + tid;   // thread = tile row
    const bool rv = r < rows;
    const int b = rv ? static_cast<int>(r / L) : 0;
    const int l = rv ? static_cast<int>(r - (long long)b * L) : 0;
    // ---- im2col row -> A (hi [, lo]); element kk = 21k + t
    uint8_t* sAlo = sA + kTileRows * kK * 2;
#pragma unroll 1
    for (int t = 0; t < kStemTaps; ++t) {
      float col[4] = {0.f, 0.f, 0.f, 0.f};
      const int p = l + t - kStemPad;
      if (rv && p >= 0 && p < L) stem_column<kIn>(in, L, b, p, col);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t off = sw128_offset(tid, 4 * t + k, kTileRows);
        const __nv_bfloat16 h = __float2bfloat16_rn(col[k]);
        *reinterpret_cast<__nv_bfloat16*>(sA + off) = h;
        if (kASplits > 1)
          *reinterpret_cast<__nv_bfloat16*>(sAlo + off) =
              __float2bfloat16_rn(col[k] - __bfloat162float(h));
      }
    }
    // zero padding kk = 84 .. 127 (rows written by their own thread)
    for (int kk = 84; kk < kK; ++kk) {
      *reinterpret_cast<__nv_bfloat16*>(sA + sw128_offset(tid, kk, kTileRows)) =
          __float2bfloat16_rn(0.f);
      if (kASplits > 1)
        *reinterpret_cast<__nv_bfloat16*>(sA + kTileRows * kK * 2 +
                                          sw128_offset(tid, kk, kTileRows)) =
            __float2bfloat16_rn(0.f);
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      uint32_t acc = 0;
      for (int term = 0; term < (kASplits > 1 ? 3 : 2); ++term) {
        const int ai = (term == 2) ? 1 : 0;
        const int bi = (term == 1) ? 1 : 0;
#pragma unroll
        for (int kk = 0; kk < kK / 16; ++kk) {
          const uint64_t da = desc_sw128(sA_addr + ai * (kTileRows * kK * 2) +
                                         (kk >> 2) * (kTileRows * 128) + (kk & 3) * 32);
          const uint64_t db = desc_sw128(sB_addr + bi * (CP * kK * 2) + (kk >> 2) * (CP * 128) +
                                         (kk & 3) * 32);
          mma_bf16(tmem, da, db, idesc, acc);
          acc = 1;
        }
      }
      mma_commit(bar);
    }
    const bool ok = mbar_wait(bar, it & 1);
    if (__syncthreads_or(!ok)) {
      if (tid == 0) atomicExch(status, kStatusTimeout);
      break;
    }
    tc_fence_after();
    // ---- bias + GELU -> X0 row
#pragma unroll 1
    for (int j = 0; j < CP / 32; ++j) {
      uint32_t d[32];
      tmem_ld32(tmem + lane_sel + j * 32, d);
      tmem_ld_wait();
      if (rv) {
        float y[32];
#pragma unroll
        for (int q = 0; q < 32; ++q) {
          const int c = j * 32 + q;
          const float z = __uint_as_float(d[q]) + (c < C ? bias[c] : 0.f);
          y[q] = (c < C) ? gelu_tanh<sizeof(act_t) == 2>(z) : 0.f;
        }
        act_t* dst = X + r * CP + j * 32;
        if constexpr (sizeof(act_t) == 2) {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            *reinterpret_cast<uint4*>(dst + q * 8) =
                make_uint4(pack_bf16x2(y[8 * q], y[8 * q + 1]), pack_bf16x2(y[8 * q + 2], y[8 * q + 3]),
                           pack_bf16x2(y[8 * q + 4], y[8 * q + 5]),
                           pack_bf16x2(y[8 * q + 6], y[8 * q + 7]));
        } else {
#pragma unroll
          for (int q = 0; q < 8; ++q)
            *reinterpret_cast<float4*>(dst + q * 4) =
                make_float4(y[4 * q], y[4 * q + 1], y[4 * q + 2], y[4 * q + 3]);
        }
      }
    }
    tc_fence_before();
    __syncthreads();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// Stem for bf16 activations with C <= 128 (CP = 128): per-example tiles of
// 128 positions (17 per 2114-bp sequence), four warpgroups per CTA, each with
// its own tile stream, A buffer and TMEM accumulator, so one group's im2col
// and epilogue overlap the other's. With the tap-major K order an im2col row
// is a contiguous window of 8-byte input columns (4 channels of one
// position): the tile's 148 columns are staged once and each row is built
// with 16-byte stores. K = 84 needs six 16-wide MMA steps. The epilogue
// (bias + GELU) writes the bf16 output tile into the A buffer in the
// 128-byte-swizzled layout of a 3-D TMA box and stores it with two TMA
// stores; positions past the end of the sequence are clipped by the tensor
// map.
namespace sm2 {
constexpr int kGroups = 4;                         // warpgroups, one tile stream each
constexpr int kThreads = 128 * kGroups;
constexpr int kCols = kTileRows + kStemTaps - 1;   // 148 staged input columns
constexpr int kKSteps = 6;                         // K = 84 -> 96
constexpr int kChunks = kKSteps * 2;               // 16-byte chunks written per row
constexpr uint32_t kW = 2 * 128 * sm::kK * 2;      // W hi | lo, 128 x 128 each
constexpr uint32_t kA = kTileRows * sm::kK * 2;    // 32 KB
__host__ __device__ constexpr uint32_t cols_bytes(int a_splits) {
  return static_cast<uint32_t>(a_splits * kCols * 8);
}
// bf16 output: four warpgroups, A buffer of a_splits x 32 KB each; fp32
// output: two warpgroups, each A region 64 KB (it also holds the fp32 output
// tile, four 32-channel boxes)
__host__ __device__ constexpr int groups_for(int out_bytes) { return out_bytes == 4 ? 2 : kGroups; }
__host__ __device__ constexpr int a_alloc(int a_splits, int out_bytes) {
  return out_bytes == 4 ? 2 : a_splits;
}
// [W hi|lo][A group 0..][cols 0..][bias][barriers]: every swizzled operand /
// TMA box starts on a 1024-byte boundary
__host__ __device__ constexpr uint32_t cols_off(int a_splits, int out_bytes = 2) {
  return kW + groups_for(out_bytes) * a_alloc(a_splits, out_bytes) * kA;
}
__host__ __device__ constexpr uint32_t cols_stride(int a_splits) {
  return (cols_bytes(a_splits) + 127) & ~127u;
}
__host__ __device__ constexpr uint32_t smem_bytes(int a_splits, int out_bytes = 2) {
  return cols_off(a_splits, out_bytes) + groups_for(out_bytes) * cols_stride(a_splits) +
         128 * 4 + 8 * (groups_for(out_bytes) + 1) + 16 + 1024;
}
static_assert(smem_bytes(1) <= 232448, "shared memory per block");
static_assert(smem_bytes(2, 4) <= 232448, "shared memory per block (fp32 output)");
static_assert(kW % 1024 == 0 && kA % 1024 == 0, "swizzled buffers need 1024-byte alignment");
}  // namespace sm2

__device__ __forceinline__ uint2 bf16x4_hi(const float (&v)[4]) {
  return make_uint2(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]));
}

// Output channels [c_off, c_off + 128) of a model with CP padded channels
// (CP = 128: one launch; CP = 256: two, c_off = 0 and 128). wpk is the packed
// [hi | lo] weight with CP rows per 128-byte-swizzled K box.
// out_t = float (fp32 mode): two warpgroups, exact GELU, the fp32 tile stored
// as four 32-channel boxes.
template <int kIn, int kASplits, typename out_t = __nv_bfloat16>
__global__ void __launch_bounds__(sm2::kThreads, 1) stem_tc_kernel(
    StemInput in, const uint8_t* __restrict__ wpk, const float* __restrict__ bias,
    const __grid_constant__ CUtensorMap tmap, int batch, int L, int C, int CP, int c_off,
    int n_tiles, int* status) {
  using namespace sm2;
  constexpr bool kF32 = sizeof(out_t) == 4;
  constexpr int kG = groups_for(sizeof(out_t));             // warpgroups
  constexpr int kAA = a_alloc(kASplits, sizeof(out_t));     // 32 KB A buffers per group
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int tid = threadIdx.x, warp = tid >> 5;
  const int g = tid >> 7, gt = tid & 127;            // warpgroup, row within the tile
  uint8_t* sB = smem;
  uint8_t* sA = smem + kW + g * kAA * kA;            // [kASplits] 128 x 128 bf16
  uint2* cols = reinterpret_cast<uint2*>(smem + cols_off(kASplits, sizeof(out_t)) +
                                         g * cols_stride(kASplits));   // [kASplits][kCols]
  float* sbias = reinterpret_cast<float*>(smem + cols_off(kASplits, sizeof(out_t)) +
                                          kG * cols_stride(kASplits));
  uint64_t* bar = reinterpret_cast<uint64_t*>(sbias + 128);    // [kG]
  uint64_t* wbar = bar + kG;                                     // W pieces arrived
  uint32_t* slot = reinterpret_cast<uint32_t*>(wbar + 1);
  if (warp == 0) tmem_alloc(slot, 128 * kG);
  if (tid == 0) {
    for (int i = 0; i < kG; ++i) mbar_init(&bar[i], 1);
    mbar_init(wbar, 1);
    mbar_init_fence();
    // rows [c_off, c_off + 128) of the hi and lo halves, both K boxes: four
    // 16 KB pieces [split][box], by bulk copies (packed weights only)
    constexpr uint32_t kPiece = 128 * 128;
    mbar_expect_tx(wbar, kW);
    for (int piece = 0; piece < static_cast<int>(kW / kPiece); ++piece) {
      const int sp = piece >> 1, kb = piece & 1;
      const size_t off = static_cast<size_t>(sp) * CP * sm::kK * 2 +
                         static_cast<size_t>(kb) * CP * 128 + static_cast<size_t>(c_off) * 128;
      bulk_load(sB + piece * kPiece, wpk + off, kPiece, wbar);
    }
  }
  if (tid < 128) sbias[tid] = c_off + tid < C ? bias[c_off + tid] : 0.f;
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  griddep_wait();                          // the previous kernel's outputs are visible
  const uint32_t tmem = *slot + g * 128;
  const uint32_t sA_addr = smem_u32(sA), sB_addr = smem_u32(sB);
  const uint32_t idesc = idesc_bf16(kTileRows, 128);
  const uint32_t lane_sel = static_cast<uint32_t>((warp & 3) * 32) << 16;
  const int tpe = (L + kTileRows - 1) / kTileRows;
  const uint32_t bar_id = 1 + g;
  uint32_t it = 0;
  bool ok = true;
  // input columns gt and gt + 128 of the group's next tile, fetched while the
  // current tile's MMAs and epilogue run
  static_assert(kCols <= 256, "two staged columns per thread");
  float pre[2][4];
  auto fetch = [&](int tile_) {
    const int b_ = tile_ / tpe;
    const int l0_ = (tile_ - b_ * tpe) * kTileRows;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int p = l0_ + gt + 128 * h - kStemPad;
#pragma unroll
      for (int k = 0; k < 4; ++k) pre[h][k] = 0.f;
      if (tile_ < n_tiles && gt + 128 * h < kCols && p >= 0 && p < L)
        stem_column<kIn>(in, L, b_, p, pre[h]);
    }
  };
  const int tile_stride = gridDim.x * kG;
  fetch(blockIdx.x * kG + g);
  // every thread (so every CTA, with or without tiles) waits for the weight
  // pieces once, while its first input columns are in flight
  ok = mbar_wait(wbar, 0);
  if (!ok && tid == 0) atomicExch(status, kStatusTimeout);
  for (int tile = blockIdx.x * kG + g; ok && tile < n_tiles; tile += tile_stride, ++it) {
    const int b = tile / tpe;
    const int l0 = (tile - b * tpe) * kTileRows;
    // ---- stage input columns l0 - 10 .. l0 + 137 (zero outside [0, L))
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int i = gt + 128 * hh;
      if (i >= kCols) continue;
      const float(&col)[4] = pre[hh];
      const uint2 h = bf16x4_hi(col);
      cols[i] = h;
      if (kASplits > 1) {
        const float lo[4] = {col[0] - __uint_as_float(h.x << 16),
                             col[1] - __uint_as_float(h.x & 0xFFFF0000u),
                             col[2] - __uint_as_float(h.y << 16),
                             col[3] - __uint_as_float(h.y & 0xFFFF0000u)};
        cols[kCols + i] = bf16x4_hi(lo);
      }
    }
    if (gt == 0) bulk_wait_read0();     // the previous output tile has left sA
    named_sync(bar_id, 128);
    // ---- im2col row gt: chunk q = taps 2q, 2q+1 (tap 21 = zero)
#pragma unroll
    for (int sp = 0; sp < kASplits; ++sp) {
      const uint2* cs = cols + sp * kCols + gt;
      uint8_t* dst = sA + sp * kA;
#pragma unroll
      for (int q = 0; q < kChunks; ++q) {
        // K column 84 (the first after the 21 taps x 4 channels) is the
        // constant 1 that multiplies the packed bias column of W
        const uint2 one = (sp == 0 && 2 * q + 1 == kStemTaps) ? make_uint2(0x3F80u, 0u)
                                                               : make_uint2(0u, 0u);
        const uint2 a = (2 * q < kStemTaps) ? cs[2 * q] : make_uint2(0u, 0u);
        const uint2 c = (2 * q + 1 < kStemTaps) ? cs[2 * q + 1] : one;
        *reinterpret_cast<uint4*>(dst + sw128_offset(gt, 8 * q, kTileRows)) =
            make_uint4(a.x, a.y, c.x, c.y);
      }
    }
    fence_async_smem();
    tc_fence_before();
    named_sync(bar_id, 128);
    if (gt == 0) {
      tc_fence_after();
      uint32_t acc = 0;
      for (int term = 0; term < (kASplits > 1 ? 3 : 2); ++term) {
        const int ai = (term == 2) ? 1 : 0;
        const int bi = (term == 1) ? 1 : 0;
#pragma unroll
        for (int kk = 0; kk < kKSteps; ++kk) {
          const uint64_t da = desc_sw128(sA_addr + ai * kA + (kk >> 2) * (kTileRows * 128) +
                                         (kk & 3) * 32);
          const uint64_t db = desc_sw128(sB_addr + bi * (kW / 2) + (kk >> 2) * (128 * 128) +
                                         (kk & 3) * 32);
          mma_bf16(tmem, da, db, idesc, acc);
          acc = 1;
        }
      }
      mma_commit(&bar[g]);
    }
    fetch(tile + tile_stride);
    ok = mbar_wait(&bar[g], it & 1);
    if (!ok) {
      if (gt == 0) atomicExch(status, kStatusTimeout);
      break;
    }
    tc_fence_after();
    if constexpr (kF32) {
      // ---- GELU -> fp32 output tile in sA: four 32-channel boxes (128-byte
      // rows, 128-byte swizzle), box j = channels [32 j, 32 j + 32)
#pragma unroll 1
      for (int j = 0; j < 4; ++j) {
        uint32_t d[32];
        tmem_ld32(tmem + lane_sel + j * 32, d);
        uint8_t* box = sA + j * kA / 2;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          float y[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) y[e] = gelu_tanh<false>(__uint_as_float(d[4 * q + e]));
          *reinterpret_cast<float4*>(box + gt * 128 + ((q ^ (gt & 7)) << 4)) =
              make_float4(y[0], y[1], y[2], y[3]);
        }
      }
      fence_async_smem();
      tc_fence_before();
      named_sync(bar_id, 128);
      if (gt == 0) {
#pragma unroll
        for (int j = 0; j < 4; ++j) tma_store_3d(&tmap, sA + j * kA / 2, c_off + 32 * j, l0, b);
        bulk_commit();
      }
    } else {
    // ---- bias + GELU -> bf16 output tile in sA (two 64-channel boxes)
#pragma unroll 1
    for (int j = 0; j < 4; ++j) {
      uint32_t d[32];
      tmem_ld32(tmem + lane_sel + j * 32, d);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t pk[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          // the bias came through the MMA; channels >= C have zero weights
          // and bias, so GELU(0) = 0 there
          pk[e] = gelu_bf16x2(__uint_as_float(d[q * 8 + 2 * e]),
                              __uint_as_float(d[q * 8 + 2 * e + 1]));
        }
        *reinterpret_cast<uint4*>(sA + sw128_offset(gt, j * 32 + q * 8, kTileRows)) =
            make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
    }
    fence_async_smem();
    tc_fence_before();
    named_sync(bar_id, 128);
    if (gt == 0) {
      tma_store_3d(&tmap, sA, c_off, l0, b);
      tma_store_3d(&tmap, sA + kTileRows * 128, c_off + 64, l0, b);
      bulk_commit();
    }
    }
  }
  if (gt == 0) bulk_wait0();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(*slot, 128 * kG);
  }
}

// ============================================================== stats
// Per-example LayerNorm statistics of the dilated depthwise conv output
// y = w0 x[l-d] + w1 x[l] + w2 x[l+d] over the (L, C) plane (upstream
// cheri.py:84-98), any activation type, one block per example (the fp32
// path; bf16 activations use stats_async_kernel below). Lanes read 8
// channels (16 B bf16 / 32 B fp32); CP/8 lanes cover one row, so a warp
// covers 256/CP rows per load instruction. Each thread accumulates sum(y) and sum(y^2)
// of one row's 8 channels in fp32 and adds them into fp64 accumulators; the
// block reduction is fp64 in a fixed order, so the result is deterministic
// and var = E[y^2] - mean^2 does not cancel catastrophically.
constexpr int kStats2Threads = 512;

template <typename act_t, int CP>
__global__ void __launch_bounds__(kStats2Threads) stats_example_kernel(
    const act_t* __restrict__ X, const float* __restrict__ convw, int dil, int L, int C,
    float eps, float2* __restrict__ stats) {
  constexpr int kLanesPerRow = CP / 8;
  constexpr int kRowsPerPass = kStats2Threads / kLanesPerRow;
  // 8 channels: one uint4 of bf16, or two float4 of fp32
  using raw_t = typename std::conditional<sizeof(act_t) == 2, uint4, Raw8f>::type;
  __shared__ double red_s[kStats2Threads / 32], red_q[kStats2Threads / 32];
  const int b = blockIdx.x;
  const int sub = threadIdx.x % kLanesPerRow;
  const int rsub = threadIdx.x / kLanesPerRow;
  const int c0 = sub * 8;
  float w0[8], w1[8], w2[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    w0[j] = convw[c0 + j];
    w1[j] = convw[CP + c0 + j];
    w2[j] = convw[2 * CP + c0 + j];
    if (c0 + j >= C) { w0[j] = 0.f; w1[j] = 0.f; w2[j] = 0.f; }
  }
  griddep_wait();                          // the previous kernel's outputs are visible
  const act_t* Xb = X + (long long)b * L * CP + c0;
  double S = 0.0, Q = 0.0;
  constexpr int kU = sizeof(act_t) == 2 ? 4 : 2;   // rows in flight per thread
  for (int l0 = rsub; l0 < L; l0 += kRowsPerPass * kU) {
    raw_t xc[kU], xl[kU], xr[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int l = l0 + u * kRowsPerPass;
      xc[u] = raw_t{}; xl[u] = raw_t{}; xr[u] = raw_t{};
      if (l < L) {
        xc[u] = ldraw<raw_t>(Xb + (long long)l * CP);
        if (l - dil >= 0) xl[u] = ldraw<raw_t>(Xb + (long long)(l - dil) * CP);
        if (l + dil < L) xr[u] = ldraw<raw_t>(Xb + (long long)(l + dil) * CP);
      }
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      float fc[8], fl[8], fr[8];
      unpack8(xc[u], fc);
      unpack8(xl[u], fl);
      unpack8(xr[u], fr);
      float s = 0.f, q = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float y = fmaf(w0[j], fl[j], fmaf(w1[j], fc[j], w2[j] * fr[j]));
        s += y;
        q = fmaf(y, y, q);
      }
      S += static_cast<double>(s);
      Q += static_cast<double>(q);
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    S += __shfl_xor_sync(0xffffffffu, S, o);
    Q += __shfl_xor_sync(0xffffffffu, Q, o);
  }
  if (lane == 0) {
    red_s[warp] = S;
    red_q[warp] = Q;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double s = 0.0, q = 0.0;
    for (int i = 0; i < kStats2Threads / 32; ++i) {
      s += red_s[i];
      q += red_q[i];
    }
    const double n = static_cast<double>(L) * static_cast<double>(C);
    const double mean = s / n;
    double var = q / n - mean * mean;
    if (var < 0.0) var = 0.0;
    stats[b] = make_float2(static_cast<float>(mean),
                           static_cast<float>(1.0 / sqrt(var + static_cast<double>(eps))));
  }
}

// Per-example statistics for bf16 activations, each element read once. Row r
// of an example belongs to the chain r = rho + k*d (rho < d); a segment is kS
// consecutive chain positions k0 .. k0+kS-1 of one chain for one 8-channel
// chunk, so the conv's left / centre / right operands of chain position k are
// positions k-1, k, k+1 of the same chain: the thread fetches the segment plus
// one halo row on each side (16 B per row, a warp covers whole rows of
// adjacent chains) and slides a three-row window through them. The rows come
// into shared memory by cp.async, double-buffered per thread: the rows of the
// thread's next segment are in flight while it sums the current one, so the
// bytes in flight per SM are not bounded by registers (2 x (kS + 2) x 16 B per
// thread, two blocks per SM). Each thread reads back only the slots it filled
// itself, so no block barrier is needed; slots are interleaved across threads
// (conflict-free 16-byte reads). The conv is fp32 on paired lanes (same
// arithmetic as the MLP producer); each segment's fp32 sums of y and y^2 fold
// into fp64 accumulators, and the block reduction is fp64 in a fixed order
// (deterministic; var = E[y^2] - mean^2 without catastrophic cancellation).
constexpr int kStatsChainThreads = 256;

template <int kS>
constexpr uint32_t stats_async_smem_bytes() {
  return static_cast<uint32_t>(2 * (kS + 2) * kStatsChainThreads * 16);
}

template <int CP, int kS>
__global__ void __launch_bounds__(kStatsChainThreads, 2) stats_async_kernel(
    const __nv_bfloat16* __restrict__ X, const float* __restrict__ convw, int dil, int L, int C,
    int n_kb, float eps, float2* __restrict__ stats) {
  constexpr int kCh = CP / 8;                       // 16-byte chunks per row
  static_assert(kStatsChainThreads % kCh == 0, "chunk count must divide the block");
  constexpr int kSegStride = kStatsChainThreads / kCh;
  constexpr int kRows = kS + 2;
  extern __shared__ uint4 slots[];                  // [buf][row][thread]
  __shared__ double red[2][kStatsChainThreads / 32];
  const int b = blockIdx.x, tid = threadIdx.x;
  const int ch = tid % kCh;
  f2 w0[4], w1[4], w2[4];
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    const int c = ch * 8 + 2 * m;
    w0[m] = f2{c < C ? convw[c] : 0.f, c + 1 < C ? convw[c + 1] : 0.f};
    w1[m] = f2{c < C ? convw[CP + c] : 0.f, c + 1 < C ? convw[CP + c + 1] : 0.f};
    w2[m] = f2{c < C ? convw[2 * CP + c] : 0.f, c + 1 < C ? convw[2 * CP + c + 1] : 0.f};
  }
  griddep_wait();                          // the previous kernel's outputs are visible
  const uint4* Xb = reinterpret_cast<const uint4*>(X + (size_t)b * L * CP) + ch;
  const int n_seg = dil * n_kb;
  auto r0_of = [&](int seg) {                       // chain position k0 = kb * kS
    const int kb = seg / dil;
    return (seg - kb * dil) + kb * kS * dil;
  };
  auto fetch = [&](int seg, int buf) {              // rows r0 + (j - 1) * d
    const int r0 = r0_of(seg);
#pragma unroll
    for (int j = 0; j < kRows; ++j) {
      const int r = r0 + (j - 1) * dil;
      const bool v = r >= 0 && r < L;
      cp_async16(&slots[(buf * kRows + j) * kStatsChainThreads + tid], Xb + (size_t)(v ? r : 0) * kCh,
                 v);
    }
    cp_async_commit();
  };
  double S = 0.0, Q = 0.0;
  int seg = tid / kCh, buf = 0;
  if (seg < n_seg) fetch(seg, 0);
  for (; seg < n_seg; seg += kSegStride, buf ^= 1) {
    const int nxt = seg + kSegStride;
    if (nxt < n_seg) {
      fetch(nxt, buf ^ 1);
      cp_async_wait<1>();                           // this segment's rows have landed
    } else {
      cp_async_wait<0>();
    }
    const int r0 = r0_of(seg);
    const uint4* sv = &slots[buf * kRows * kStatsChainThreads + tid];
    uint4 vl = sv[0], vc = sv[kStatsChainThreads];
    f2 sy[4], sq[4];
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      sy[m] = f2{0.f, 0.f};
      sq[m] = f2{0.f, 0.f};
    }
#pragma unroll
    for (int j = 1; j <= kS; ++j) {
      const uint4 vr = sv[(j + 1) * kStatsChainThreads];
      if (r0 + (j - 1) * dil < L) {
        const uint32_t* pl = reinterpret_cast<const uint32_t*>(&vl);
        const uint32_t* pc = reinterpret_cast<const uint32_t*>(&vc);
        const uint32_t* pr = reinterpret_cast<const uint32_t*>(&vr);
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const f2 xl{__uint_as_float(pl[m] << 16), __uint_as_float(pl[m] & 0xFFFF0000u)};
          const f2 xc{__uint_as_float(pc[m] << 16), __uint_as_float(pc[m] & 0xFFFF0000u)};
          const f2 xr{__uint_as_float(pr[m] << 16), __uint_as_float(pr[m] & 0xFFFF0000u)};
          const f2 y = fma2(w0[m], xl, fma2(w1[m], xc, mul2(w2[m], xr)));
          sy[m] = f2{sy[m].x + y.x, sy[m].y + y.y};
          sq[m] = fma2(y, y, sq[m]);
        }
      }
      vl = vc;
      vc = vr;
    }
    const float ts = ((sy[0].x + sy[0].y) + (sy[1].x + sy[1].y)) +
                     ((sy[2].x + sy[2].y) + (sy[3].x + sy[3].y));
    const float tq = ((sq[0].x + sq[0].y) + (sq[1].x + sq[1].y)) +
                     ((sq[2].x + sq[2].y) + (sq[3].x + sq[3].y));
    S += static_cast<double>(ts);
    Q += static_cast<double>(tq);
  }
  const int warp = tid >> 5, lane = tid & 31;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    S += __shfl_xor_sync(0xffffffffu, S, o);
    Q += __shfl_xor_sync(0xffffffffu, Q, o);
  }
  if (lane == 0) {
    red[0][warp] = S;
    red[1][warp] = Q;
  }
  __syncthreads();
  if (tid == 0) {
    double ss = 0.0, qq = 0.0;
    for (int i = 0; i < kStatsChainThreads / 32; ++i) {
      ss += red[0][i];
      qq += red[1][i];
    }
    const double n = static_cast<double>(L) * static_cast<double>(C);
    const double mean = ss / n;
    double var = qq / n - mean * mean;
    if (var < 0.0) var = 0.0;
    stats[b] = make_float2(static_cast<float>(mean),
                           static_cast<float>(1.0 / sqrt(var + static_cast<double>(eps))));
  }
}

// ============================================================== MLP
// One Cheri Block update for 128-row tiles of the flattened (B*L) rows:
//   A1 = bf16((conv(X) - mean) * rstd)            (built by all threads)
//   D1 = A1 * W1^T                                (tcgen05, TMEM, fp32)
//   A2 = bf16(gelu(D1))                           (TMEM -> registers -> smem)
//   D2 = A2 * (rs * W2)^T                         (tcgen05, TMEM, fp32)
//   X_out = X + D2
// (upstream cheri.py:1072-1082; the Triton equivalent is
// _fwd_inf_norm_mlp_kernel, cheri.py:594-669). Persistent: one CTA per SM,
// W1/W2 resident in shared memory for the whole launch.
struct MlpArgs {
  const void* X_in;
  void* X_out;
  const float2* stats;
  const uint8_t* w1;     // packed bf16 W1 tile (HP x CP, swizzled)
  const uint8_t* w2;     // packed bf16 rs*W2 tile (CP x HP, swizzled)
  const float* convw;    // (3, CP) fp32
  int dil;
  int L;
  int C;
  long long rows;        // B * L
  int n_tiles;           // flattened 128-row tiles; per-example tiles in mlp_ws_kernel
  int tpe;               // mlp_ws_kernel: 128-row tiles per example (ceil(L / 128))
  int HP;                // mlp_stream_kernel: padded hidden width
  int* status;
};

template <int CP, int HP>
struct MlpSmem {
  static constexpr uint32_t kW1 = 0;
  static constexpr uint32_t kW2 = kW1 + HP * CP * 2;
  static constexpr uint32_t kA2 = kW2 + CP * HP * 2;   // A1 aliases the start of A2
  static constexpr uint32_t kBar = kA2 + kTileRows * HP * 2;
  static constexpr uint32_t kSlot = kBar + 16;
  static constexpr uint32_t kBytes = kSlot + 16;
  static constexpr uint32_t kAlloc = kBytes + 1024;      // room to align the base to 1024
};

template <typename act_t, int CP, int HP, bool kFastGelu>
__global__ void __launch_bounds__(128, 1) mlp_kernel(MlpArgs a) {
  static_assert(CP % 64 == 0 && HP % 64 == 0 && HP >= CP && HP <= 256 && CP <= 128,
                "tile shapes");
  using S = MlpSmem<CP, HP>;
  constexpr int CPL = CP / 32;
  constexpr uint32_t kTmemCols = 512;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sW1 = smem + S::kW1;
  uint8_t* sW2 = smem + S::kW2;
  uint8_t* sA = smem + S::kA2;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kBar);
  uint32_t* slot = reinterpret_cast<uint32_t*>(smem + S::kSlot);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const act_t* Xi = static_cast<const act_t*>(a.X_in);
  act_t* Xo = static_cast<act_t*>(a.X_out);

  if (warp == 0) tmem_alloc(slot, kTmemCols);
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    mbar_init_fence();
  }
  {  // weights -> shared memory (already in the swizzled operand layout)
    const uint4* g1 = reinterpret_cast<const uint4*>(a.w1);
    const uint4* g2 = reinterpret_cast<const uint4*>(a.w2);
    uint4* s1 = reinterpret_cast<uint4*>(sW1);
    uint4* s2 = reinterpret_cast<uint4*>(sW2);
    for (int i = tid; i < HP * CP * 2 / 16; i += blockDim.x) s1[i] = g1[i];
    for (int i = tid; i < CP * HP * 2 / 16; i += blockDim.x) s2[i] = g2[i];
  }
  const int c0 = lane * CPL;
  float cw0[CPL], cw1[CPL], cw2[CPL];
#pragma unroll
  for (int j = 0; j < CPL; ++j) {
    cw0[j] = a.convw[c0 + j];
    cw1[j] = a.convw[CP + c0 + j];
    cw2[j] = a.convw[2 * CP + c0 + j];
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *slot;
  const uint32_t tD1 = tmem;         // columns [0, HP)
  const uint32_t tD2 = tmem + HP;    // columns [HP, HP + CP)
  const uint32_t lane_sel = static_cast<uint32_t>(warp * 32) << 16;
  const uint32_t sA_addr = smem_u32(sA), sW1_addr = smem_u32(sW1), sW2_addr = smem_u32(sW2);
  constexpr uint32_t kIdesc1 = idesc_bf16(kTileRows, HP);
  constexpr uint32_t kIdesc2 = idesc_bf16(kTileRows, CP);

  bool failed = false;
  uint32_t it = 0;
  for (int tile = blockIdx.x; tile < a.n_tiles; tile += gridDim.x, ++it) {
    const long long row0 = (long long)tile * kTileRows;
    // ---- A1: conv + LayerNorm, bf16, swizzled (warp w builds rows 32w..32w+31)
    for (int i = 0; i < 32; ++i) {
      const int rl = warp * 32 + i;
      const long long r = row0 + rl;
      float v[CPL];
#pragma unroll
      for (int j = 0; j < CPL; ++j) v[j] = 0.f;
      if (r < a.rows) {
        const int n = static_cast<int>(r / a.L);
        const int l = static_cast<int>(r - (long long)n * a.L);
        const float2 st = a.stats[n];
        float xc[CPL], xl[CPL], xr[CPL];
#pragma unroll
        for (int j = 0; j < CPL; ++j) { xl[j] = 0.f; xr[j] = 0.f; }
        Vec<act_t, CPL>::load(Xi + r * CP + c0, xc);
        if (l - a.dil >= 0) Vec<act_t, CPL>::load(Xi + (r - a.dil) * CP + c0, xl);
        if (l + a.dil < a.L) Vec<act_t, CPL>::load(Xi + (r + a.dil) * CP + c0, xr);
#pragma unroll
        for (int j = 0; j < CPL; ++j) {
          const float y = fmaf(cw0[j], xl[j], fmaf(cw1[j], xc[j], cw2[j] * xr[j]));
          v[j] = (c0 + j < a.C) ? (y - st.x) * st.y : 0.f;
        }
      }
      const uint32_t off = sw128_offset(rl, c0, kTileRows);
      if constexpr (CPL == 4) {
        *reinterpret_cast<uint2*>(sA + off) =
            make_uint2(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]));
      } else {
        *reinterpret_cast<uint32_t*>(sA + off) = pack_bf16x2(v[0], v[1]);
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    // ---- GEMM1
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int k = 0; k < CP / 16; ++k) {
        const uint64_t da = desc_sw128(sA_addr + (k >> 2) * (kTileRows * 128) + (k & 3) * 32);
        const uint64_t db = desc_sw128(sW1_addr + (k >> 2) * (HP * 128) + (k & 3) * 32);
        mma_bf16(tD1, da, db, kIdesc1, k > 0 ? 1u : 0u);
      }
      mma_commit(&bars[0]);
    }
    bool ok = mbar_wait(&bars[0], it & 1);
    if (__syncthreads_or(!ok)) { failed = true; break; }
    tc_fence_after();
    // ---- GELU: TMEM D1 -> bf16 A2 (thread = row 32*warp + lane)
    {
      const int rl = warp * 32 + lane;
#pragma unroll 1
      for (int j = 0; j < HP / 32; ++j) {
        uint32_t r[32];
        tmem_ld32(tD1 + lane_sel + j * 32, r);
        tmem_ld_wait();
        uint32_t p[16];
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const float g0 = gelu_tanh<kFastGelu>(__uint_as_float(r[2 * q]));
          const float g1 = gelu_tanh<kFastGelu>(__uint_as_float(r[2 * q + 1]));
          p[q] = pack_bf16x2(g0, g1);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t off = sw128_offset(rl, j * 32 + q * 8, kTileRows);
          *reinterpret_cast<uint4*>(sA + off) =
              make_uint4(p[4 * q], p[4 * q + 1], p[4 * q + 2], p[4 * q + 3]);
        }
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    // ---- GEMM2
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int k = 0; k < HP / 16; ++k) {
        const uint64_t da = desc_sw128(sA_addr + (k >> 2) * (kTileRows * 128) + (k & 3) * 32);
        const uint64_t db = desc_sw128(sW2_addr + (k >> 2) * (CP * 128) + (k & 3) * 32);
        mma_bf16(tD2, da, db, kIdesc2, k > 0 ? 1u : 0u);
      }
      mma_commit(&bars[1]);
    }
    ok = mbar_wait(&bars[1], it & 1);
    if (__syncthreads_or(!ok)) { failed = true; break; }
    tc_fence_after();
    // ---- residual: X_out = X_in + D2 (thread = row)
    {
      const long long r = row0 + warp * 32 + lane;
#pragma unroll 1
      for (int j = 0; j < CP / 32; ++j) {
        uint32_t d[32];
        tmem_ld32(tD2 + lane_sel + j * 32, d);
        tmem_ld_wait();
        if (r < a.rows) {
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            float x[4];
            Vec<act_t, 4>::load(Xi + r * CP + j * 32 + q * 4, x);
#pragma unroll
            for (int e = 0; e < 4; ++e) x[e] += __uint_as_float(d[q * 4 + e]);
            Vec<act_t, 4>::store(Xo + r * CP + j * 32 + q * 4, x);
          }
        }
      }
    }
    tc_fence_before();
    __syncthreads();
  }
  if (failed && tid == 0) atomicExch(a.status, kStatusTimeout);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ============================================================== MLP, streamed weights
// Cheri Block update for wide models (C up to 256, H up to 512), whose W1 and
// W2 do not fit in shared memory together. Per 128-row tile (one CTA per SM,
// persistent, 8 warps):
//   A1 = bf16((conv(X) - mean) * rstd)      -> shared memory (K-major, swizzled)
//   for each chunk of 64 hidden units hc:
//     D1 = A1 * W1[hc]^T                    (tcgen05, TMEM, K = CP)
//     A2 = bf16(gelu(D1))                   -> shared memory
//     D2 (+)= A2 * W2[:, hc]^T              (tcgen05, TMEM, K = 64)
//   X_out = X + D2
// The weight chunks (W1 rows [64 hc, 64 hc + 64): CP/64 pieces of 8 KB; W2
// columns of chunk hc: one CP x 128-byte piece, both straight from the packed
// 128-byte-swizzled layout) stream in by 1-D bulk copies into two buffers, one
// chunk ahead. Upstream cheri.py:1072-1082.
template <int CP>
struct StreamSmem {
  static constexpr uint32_t kA1 = 0;                          // CP/64 x (128 x 128 B)
  static constexpr uint32_t kWBuf = static_cast<uint32_t>(CP) * 256;   // W1 chunk + W2 chunk
  static constexpr uint32_t kW = kA1 + static_cast<uint32_t>(CP) * 256;
  static constexpr uint32_t kA2 = kW + 2 * kWBuf;             // 128 x 64 bf16
  static constexpr uint32_t kBars = kA2 + 128 * 128;
  static constexpr uint32_t kSlot = kBars + 4 * 8;
  static constexpr uint32_t kAlloc = kSlot + 16 + 1024;
  static_assert(kAlloc <= 232448, "shared memory per block");
};

template <typename act_t, int CP, bool kFastGelu>
__global__ void __launch_bounds__(256, 1) mlp_stream_kernel(MlpArgs a) {
  static_assert(CP == 64 || CP == 128 || CP == 256, "channel width");
  using S = StreamSmem<CP>;
  const int HP = a.HP;                               // padded hidden width, multiple of 64
  const int kChunks = HP / 64;
  constexpr int CPL = CP / 32;                       // channels per lane when building A1
  constexpr uint32_t kTmemCols = (CP + 64 <= 256) ? 256 : 512;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA1 = smem + S::kA1;
  uint8_t* sW = smem + S::kW;
  uint8_t* sA2 = smem + S::kA2;
  uint64_t* wfull = reinterpret_cast<uint64_t*>(smem + S::kBars);   // [2]
  uint64_t* mbar = wfull + 2;
  uint32_t* slot = reinterpret_cast<uint32_t*>(smem + S::kSlot);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const act_t* Xi = static_cast<const act_t*>(a.X_in);
  act_t* Xo = static_cast<act_t*>(a.X_out);

  if (warp == 0) tmem_alloc(slot, kTmemCols);
  if (tid == 0) {
    mbar_init(&wfull[0], 1);
    mbar_init(&wfull[1], 1);
    mbar_init(mbar, 1);
    mbar_init_fence();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *slot;
  const uint32_t tD2 = tmem;                         // columns [0, CP)
  const uint32_t tD1 = tmem + CP;                    // columns [CP, CP + 64)
  const uint32_t lane_sel = static_cast<uint32_t>((warp & 3) * 32) << 16;
  const uint32_t sA1_addr = smem_u32(sA1), sW_addr = smem_u32(sW), sA2_addr = smem_u32(sA2);
  constexpr uint32_t kIdesc1 = idesc_bf16(kTileRows, 64);
  constexpr uint32_t kIdesc2 = idesc_bf16(kTileRows, CP);
  const int n_my = (a.n_tiles > (int)blockIdx.x)
                       ? (a.n_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x
                       : 0;
  const long long total = (long long)n_my * kChunks;   // weight chunks this CTA uses
  // weight chunk g (hidden chunk g % kChunks) -> buffer g & 1
  auto load_w = [&](long long g) {
    const int hc = static_cast<int>(g % kChunks), buf = static_cast<int>(g & 1);
    uint8_t* dst = sW + buf * S::kWBuf;
    mbar_expect_tx(&wfull[buf], S::kWBuf);
#pragma unroll
    for (int kb = 0; kb < CP / 64; ++kb)
      bulk_load(dst + kb * 8192, a.w1 + ((size_t)kb * HP + 64 * hc) * 128, 8192, &wfull[buf]);
    bulk_load(dst + (CP / 64) * 8192, a.w2 + (size_t)hc * CP * 128, CP * 128, &wfull[buf]);
  };
  if (tid == 0) {
    if (total > 0) load_w(0);
    if (total > 1) load_w(1);
  }
  float cw0[CPL], cw1[CPL], cw2[CPL];
  const int c0 = lane * CPL;
#pragma unroll
  for (int j = 0; j < CPL; ++j) {
    cw0[j] = a.convw[c0 + j];
    cw1[j] = a.convw[CP + c0 + j];
    cw2[j] = a.convw[2 * CP + c0 + j];
  }
  bool ok = true;
  uint32_t mph = 0;                                  // MMA barrier completions so far
  for (int it = 0; it < n_my && ok; ++it) {
    const long long row0 = (long long)((int)blockIdx.x + it * (int)gridDim.x) * kTileRows;
    // ---- A1: conv + LayerNorm (warp w builds rows 16w .. 16w + 15)
    for (int i = 0; i < 16; ++i) {
      const int rl = warp * 16 + i;
      const long long r = row0 + rl;
      float v[CPL];
#pragma unroll
      for (int j = 0; j < CPL; ++j) v[j] = 0.f;
      if (r < a.rows) {
        const int n = static_cast<int>(r / a.L);
        const int l = static_cast<int>(r - (long long)n * a.L);
        const float2 st = a.stats[n];
        float xc[CPL], xl[CPL], xr[CPL];
#pragma unroll
        for (int j = 0; j < CPL; ++j) { xl[j] = 0.f; xr[j] = 0.f; }
        Vec<act_t, CPL>::load(Xi + r * CP + c0, xc);
        if (l - a.dil >= 0) Vec<act_t, CPL>::load(Xi + (r - a.dil) * CP + c0, xl);
        if (l + a.dil < a.L) Vec<act_t, CPL>::load(Xi + (r + a.dil) * CP + c0, xr);
#pragma unroll
        for (int j = 0; j < CPL; ++j) {
          const float y = fmaf(cw0[j], xl[j], fmaf(cw1[j], xc[j], cw2[j] * xr[j]));
          v[j] = (c0 + j < a.C) ? (y - st.x) * st.y : 0.f;
        }
      }
#pragma unroll
      for (int j = 0; j < CPL; j += 2)
        *reinterpret_cast<uint32_t*>(sA1 + sw128_offset(rl, c0 + j, kTileRows)) =
            pack_bf16x2(v[j], v[j + 1]);
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    for (int hc = 0; hc < kChunks && ok; ++hc) {
      const long long g = (long long)it * kChunks + hc;
      const int buf = static_cast<int>(g & 1);
      const uint32_t w1_addr = sW_addr + buf * S::kWBuf;
      const uint32_t w2_addr = w1_addr + (CP / 64) * 8192;
      // ---- GEMM1: D1 = A1 * W1[hc]^T
      if (tid == 0) {
        ok = mbar_wait(&wfull[buf], static_cast<uint32_t>((g >> 1) & 1));
        if (ok) {
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < CP / 16; ++k) {
            const uint64_t da = desc_sw128(sA1_addr + (k >> 2) * (kTileRows * 128) + (k & 3) * 32);
            const uint64_t db = desc_sw128(w1_addr + (k >> 2) * 8192 + (k & 3) * 32);
            mma_bf16(tD1, da, db, kIdesc1, k > 0 ? 1u : 0u);
          }
          mma_commit(mbar);
        }
      }
      if (__syncthreads_or(!ok)) { ok = false; break; }
      ok = mbar_wait(mbar, mph & 1);
      ++mph;
      if (__syncthreads_or(!ok)) { ok = false; break; }
      tc_fence_after();
      // ---- GELU: thread (row, half) -> 32 hidden units -> A2 (bf16, swizzled)
      {
        const int rl = (warp & 3) * 32 + lane, half = warp >> 2;
        uint32_t r[32];
        tmem_ld32(tD1 + lane_sel + half * 32, r);
        uint32_t p[16];
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          if constexpr (kFastGelu) {
            p[q] = gelu_bf16x2(__uint_as_float(r[2 * q]), __uint_as_float(r[2 * q + 1]));
          } else {
            p[q] = pack_bf16x2(gelu_tanh<false>(__uint_as_float(r[2 * q])),
                               gelu_tanh<false>(__uint_as_float(r[2 * q + 1])));
          }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q)
          *reinterpret_cast<uint4*>(sA2 + sw128_offset(rl, half * 32 + q * 8, kTileRows)) =
              make_uint4(p[4 * q], p[4 * q + 1], p[4 * q + 2], p[4 * q + 3]);
      }
      fence_async_smem();
      tc_fence_before();
      __syncthreads();
      // ---- GEMM2: D2 (+)= A2 * W2[:, hc]^T; then buffer `buf` is free again
      if (tid == 0) {
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t da = desc_sw128(sA2_addr + (k & 3) * 32);
          const uint64_t db = desc_sw128(w2_addr + (k & 3) * 32);
          mma_bf16(tD2, da, db, kIdesc2, (hc > 0 || k > 0) ? 1u : 0u);
        }
        mma_commit(mbar);
      }
      ok = mbar_wait(mbar, mph & 1);
      ++mph;
      if (__syncthreads_or(!ok)) { ok = false; break; }
      tc_fence_after();
      if (tid == 0 && g + 2 < total) load_w(g + 2);
    }
    if (!ok) break;
    // ---- residual: X_out = X_in + D2 (thread = row, half of the channels)
    {
      const int rl = (warp & 3) * 32 + lane, half = warp >> 2;
      const long long r = row0 + rl;
#pragma unroll 1
      for (int j = 0; j < CP / 64; ++j) {
        const int cb = half * (CP / 2) + j * 32;
        uint32_t d[32];
        tmem_ld32(tD2 + lane_sel + cb, d);
        if (r < a.rows) {
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            float x[4];
            Vec<act_t, 4>::load(Xi + r * CP + cb + q * 4, x);
#pragma unroll
            for (int e = 0; e < 4; ++e) x[e] += __uint_as_float(d[q * 4 + e]);
            Vec<act_t, 4>::store(Xo + r * CP + cb + q * 4, x);
          }
        }
      }
    }
    tc_fence_before();
    __syncthreads();
  }
  if (!ok && tid == 0) atomicExch(a.status, kStatusTimeout);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ============================================================== MLP, wide (C = 256), bf16
// Warp-specialised persistent Cheri Block update for n_filters 256 in bf16
// mode (any hidden width HP = 64 k <= 512), one CTA per SM, 128-row tiles of
// the flattened (B * L) rows. W1 and W2 (up to 512 KB) stream from L2 in
// 32 KB stages, one per MMA group, so the tile's GEMMs are chunked along the
// hidden dimension (64 units per chunk c):
//   G1(c): D1[c & 1] = A1 * W1[c]^T     (A1 in shared memory, K = 256, N = 64)
//   GELU : A2(c) = bf16(gelu(D1[c & 1])) written back into D1's columns
//   G2(c): D2 (+)= A2(c) * W2[:, c]^T   (A2 from TMEM, K = 64, N = 256)
// issued as G1(0) G1(1) G2(0) G1(2) G2(1) G1(3) ..., so the GELU of chunk c
// overlaps G1(c + 1); G1(c + 2) overwrites D1[c & 1] only after G2(c) read it
// (MMAs of one thread execute in order). Roles (22 warps):
//   warps 0-7   producer : A1(t + 1) = bf16((conv(X) - mean) * rstd / 2) into
//                          the other of two shared-memory A1 buffers; lane =
//                          8 channels of a row (coalesced 512-byte rows)
//   warps 8-15  GELU     : lane quarter x column half of each D1 chunk
//   warps 16-19 residual : thread = row; stages the tile's input row as bf16
//                          in TMEM ahead of time, then X_out = X + bf16(D2)
//   warp 20     MMA      : one thread issues every tcgen05.mma
//   warp 21     TMA      : one thread streams the weight stages
// TMEM: D2 [0,256) | D1[0] [256,320) | D1[1] [320,384) | X stage [384,512).
// A1 carries the factor 1/2 the GELU of D1/2 expects (gelu_half_bf16x2), as
// in the default-width kernel. Upstream cheri.py:1072-1082.
namespace wd {
constexpr int kCP = 256;
constexpr int kProducerWarps = 8, kGeluWarps = 8, kResidualWarps = 4;
constexpr int kGeluWarp0 = kProducerWarps;                      // 8
constexpr int kResidualWarp0 = kGeluWarp0 + kGeluWarps;         // 16
constexpr int kMmaWarp = kResidualWarp0 + kResidualWarps;       // 20
constexpr int kTmaWarp = kMmaWarp + 1;                          // 21
constexpr int kThreads = (kTmaWarp + 1) * 32;                   // 704
constexpr uint32_t kA1Bytes = 128 * kCP * 2;                    // 64 KB: 4 K boxes of 16 KB
constexpr uint32_t kStage = 32768;                              // one weight stage
constexpr int kStages = 3;
constexpr uint32_t kA1 = 0;                                     // 2 A1 buffers
constexpr uint32_t kW = 2 * kA1Bytes;                           // weight ring
enum Bar : int { A1_FULL0 = 0, A1_FULL1, A1_EMPTY0, A1_EMPTY1, W_FULL0, W_EMPTY0 = W_FULL0 + kStages,
                 D1_FULL0 = W_EMPTY0 + kStages, D1_FULL1, A2_FULL0, A2_FULL1, D2_FULL, D2_EMPTY,
                 kNumBars };
constexpr uint32_t kBars = kW + kStages * kStage;
constexpr uint32_t kSlot = kBars + kNumBars * 8;
constexpr uint32_t kAbort = kSlot + 4;
constexpr uint32_t kAlloc = kAbort + 4 + 1024;
static_assert(kAlloc <= 232448, "shared memory per block");
constexpr uint32_t kD2Col = 0, kD1Col = 256, kXsCol = 384;
}  // namespace wd

__global__ void __launch_bounds__(wd::kThreads, 1) mlp_wide_kernel(MlpArgs a) {
  using namespace wd;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBars);
  uint32_t* slot = reinterpret_cast<uint32_t*>(smem + kSlot);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kAbort);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kChunks = a.HP / 64;
  const __nv_bfloat16* Xi = static_cast<const __nv_bfloat16*>(a.X_in);
  __nv_bfloat16* Xo = static_cast<__nv_bfloat16*>(a.X_out);

  if (warp == kMmaWarp) tmem_alloc(slot, 512);
  if (tid == 0) {
    for (int i = 0; i < kNumBars; ++i) {
      uint32_t count = 1;                           // commits, TMA transactions
      if (i == A1_FULL0 || i == A1_FULL1) count = kProducerWarps;
      else if (i == A2_FULL0 || i == A2_FULL1) count = kGeluWarps;
      else if (i == D2_EMPTY) count = kResidualWarps;
      mbar_init(&bars[i], count);
    }
    *abort_flag = 0;
    mbar_init_fence();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  griddep_wait();                          // the previous kernel's outputs are visible
  const uint32_t tmem = *slot;
  const int n_my = (a.n_tiles > static_cast<int>(blockIdx.x))
                       ? (a.n_tiles - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                             static_cast<int>(gridDim.x)
                       : 0;
  const int c_total = n_my * kChunks;               // hidden chunks this CTA processes
  auto row0_of = [&](int it) -> long long {
    return static_cast<long long>(static_cast<int>(blockIdx.x) + it * static_cast<int>(gridDim.x)) *
           kTileRows;
  };

  if (warp < kProducerWarps) {
    // ------------------------------------------------------------ producer
    // conv weights of this lane's channels [8 lane, 8 lane + 8) as bf16x2
    // pairs per tap (zero past C); pairs past C are also masked to 0 in A1
    const int c0 = 8 * lane;
    uint32_t w0[4], w1[4], w2[4], cmask[4];
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int c = c0 + 2 * m;
      auto wv = [&](int t, int cc) { return cc < a.C ? a.convw[t * kCP + cc] : 0.f; };
      w0[m] = pack_bf16x2(wv(0, c), wv(0, c + 1));
      w1[m] = pack_bf16x2(wv(1, c), wv(1, c + 1));
      w2[m] = pack_bf16x2(wv(2, c), wv(2, c + 1));
      cmask[m] = (c < a.C ? 0x0000FFFFu : 0u) | (c + 1 < a.C ? 0xFFFF0000u : 0u);
    }
    const uint32_t box_off = static_cast<uint32_t>(lane >> 3) * 16384u;   // K box of the lane
    const int q = lane & 7;                                               // 16-byte chunk in the box row
    bool ok = true;
    for (int it = 0; it < n_my && ok; ++it) {
      const int buf = it & 1;
      ok = mbar_wait_abortable(&bars[A1_EMPTY0 + buf], ((it >> 1) & 1) ^ 1, abort_flag);
      if (!ok) break;
      uint8_t* sA1 = smem + kA1 + buf * kA1Bytes + box_off;
      const long long row0 = row0_of(it);
      constexpr int kU = 3;                                  // rows in flight per warp
      for (int i0 = warp; i0 < kTileRows; i0 += kProducerWarps * kU) {
        uint4 xl[kU], xc[kU], xr[kU];
        float2 st[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int rl = i0 + u * kProducerWarps;
          const long long r = row0 + rl;
          xl[u] = make_uint4(0u, 0u, 0u, 0u);
          xc[u] = xl[u];
          xr[u] = xl[u];
          st[u] = make_float2(0.f, 0.f);
          if (rl < kTileRows && r < a.rows) {
            const int n = static_cast<int>(r / a.L);
            const int l = static_cast<int>(r - static_cast<long long>(n) * a.L);
            st[u] = a.stats[n];
            const uint4* xp = reinterpret_cast<const uint4*>(Xi + r * kCP + c0);
            xc[u] = __ldg(xp);
            if (l - a.dil >= 0) xl[u] = __ldg(xp - static_cast<long long>(a.dil) * (kCP / 8));
            if (l + a.dil < a.L) xr[u] = __ldg(xp + static_cast<long long>(a.dil) * (kCP / 8));
          }
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int rl = i0 + u * kProducerWarps;
          if (rl >= kTileRows) break;
          // A1 = (y - mean) * rstd / 2 in bf16x2: y = w0 x[l-d] + w1 x[l] + w2 x[l+d]
          const uint32_t scale_b = pack_bf16x2(0.5f * st[u].y, 0.5f * st[u].y);
          const uint32_t shift_b = pack_bf16x2(-0.5f * st[u].x * st[u].y, -0.5f * st[u].x * st[u].y);
          const uint32_t* pl = &xl[u].x;
          const uint32_t* pc = &xc[u].x;
          const uint32_t* pr = &xr[u].x;
          uint32_t o[4];
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            uint32_t y = bf2_mul(w2[m], pr[m]);
            y = bf2_fma(w1[m], pc[m], y);
            y = bf2_fma(w0[m], pl[m], y);
            o[m] = bf2_fma(y, scale_b, shift_b) & cmask[m];
          }
          *reinterpret_cast<uint4*>(sA1 + rl * 128 + ((q ^ (rl & 7)) << 4)) =
              make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
      fence_async_smem();                          // generic writes -> MMA (async proxy)
      mbar_arrive_warp(&bars[A1_FULL0 + buf]);
    }
  } else if (warp < kResidualWarp0) {
    // ------------------------------------------------------------ GELU
    const int quarter = warp & 3, half = (warp - kGeluWarp0) >> 2;
    const uint32_t lane_sel = static_cast<uint32_t>(quarter * 32) << 16;
    for (int c = 0; c < c_total; ++c) {
      const int b = c & 1;
      if (!mbar_wait_abortable(&bars[D1_FULL0 + b], (c >> 1) & 1, abort_flag)) break;
      tc_fence_after();
      // columns [32 half, 32 half + 32) of the chunk, packed in place into
      // [32 half, 32 half + 16) (already read by this warp)
      const uint32_t base = tmem + lane_sel + kD1Col + b * 64 + half * 32;
      uint32_t r[32];
      tmem_ld32(base, r);
      uint32_t p[16];
#pragma unroll
      for (int k = 0; k < 16; ++k)
        p[k] = gelu_half_bf16x2(__uint_as_float(r[2 * k]), __uint_as_float(r[2 * k + 1]));
      tmem_st16(base, p);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive_warp(&bars[A2_FULL0 + b]);
    }
  } else if (warp < kMmaWarp) {
    // ------------------------------------------------------------ residual
    const int quarter = warp & 3;
    const int rl = quarter * 32 + lane;
    const uint32_t lane_sel = static_cast<uint32_t>(quarter * 32) << 16;
    for (int it = 0; it < n_my; ++it) {
      const long long r = row0_of(it) + rl;
      const bool rv = r < a.rows;
      // stage this row's input in TMEM (bf16 pairs: 256 channels -> 128
      // columns), long before D2 is ready
      const uint4* xp = reinterpret_cast<const uint4*>(Xi + (rv ? r : 0) * kCP);
#pragma unroll 1
      for (int g = 0; g < 8; ++g) {                 // 32 channels = 4 x 16 bytes -> 16 columns
        uint32_t v[16];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint4 a0 = rv ? __ldg(xp + g * 4 + k) : make_uint4(0u, 0u, 0u, 0u);
          v[4 * k] = a0.x;
          v[4 * k + 1] = a0.y;
          v[4 * k + 2] = a0.z;
          v[4 * k + 3] = a0.w;
        }
        tmem_st16(tmem + lane_sel + kXsCol + 16 * g, v);
      }
      tmem_st_wait();
      if (!mbar_wait_abortable(&bars[D2_FULL], it & 1, abort_flag)) break;
      tc_fence_after();
      uint4* op = reinterpret_cast<uint4*>(Xo + r * kCP);
#pragma unroll 1
      for (int g = 0; g < 8; ++g) {                 // 32 output channels per step
        uint32_t d[32], x[16];
        tmem_ld32(tmem + lane_sel + kD2Col + 32 * g, d);
        tmem_ld16(tmem + lane_sel + kXsCol + 16 * g, x);
        if (g == 7) {
          tc_fence_before();
          mbar_arrive_warp(&bars[D2_EMPTY]);         // D2 fully read
        }
        uint32_t o[16];
#pragma unroll
        for (int k = 0; k < 16; ++k)
          o[k] = bf2_add(x[k], pack_bf16x2(__uint_as_float(d[2 * k]), __uint_as_float(d[2 * k + 1])));
        if (rv) {
#pragma unroll
          for (int k = 0; k < 4; ++k)
            op[4 * g + k] = make_uint4(o[4 * k], o[4 * k + 1], o[4 * k + 2], o[4 * k + 3]);
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && c_total > 0) {
      const uint32_t sW = smem_u32(smem + kW);
      constexpr uint32_t kIdesc1 = idesc_bf16(kTileRows, 64);
      constexpr uint32_t kIdesc2 = idesc_bf16(kTileRows, kCP);
      uint32_t k_stage = 0;                          // weight stages consumed
      bool ok = true;
      auto stage_in = [&]() -> uint32_t {            // wait for the next weight stage
        const uint32_t s = k_stage % kStages;
        ok = ok && mbar_wait_abortable(&bars[W_FULL0 + s], (k_stage / kStages) & 1, abort_flag);
        return s;
      };
      auto g1 = [&](int c) {
        const int t = c / kChunks, j = c - t * kChunks;
        if (j == 0) ok = ok && mbar_wait_abortable(&bars[A1_FULL0 + (t & 1)], (t >> 1) & 1, abort_flag);
        const uint32_t s = stage_in();
        if (!ok) return;
        tc_fence_after();
        const uint32_t sA = smem_u32(smem + kA1 + (t & 1) * kA1Bytes);
        const uint32_t sB = sW + s * kStage;
        const uint32_t d = tmem + kD1Col + (c & 1) * 64;
#pragma unroll
        for (int k = 0; k < kCP / 16; ++k)
          mma_bf16(d, desc_sw128(sA + (k >> 2) * 16384 + (k & 3) * 32),
                   desc_sw128(sB + (k >> 2) * 8192 + (k & 3) * 32), kIdesc1, k > 0 ? 1u : 0u);
        mma_commit(&bars[W_EMPTY0 + s]);
        mma_commit(&bars[D1_FULL0 + (c & 1)]);
        if (j == kChunks - 1) mma_commit(&bars[A1_EMPTY0 + (t & 1)]);
        ++k_stage;
      };
      auto g2 = [&](int c) {
        const int t = c / kChunks, j = c - t * kChunks;
        ok = ok && mbar_wait_abortable(&bars[A2_FULL0 + (c & 1)], (c >> 1) & 1, abort_flag);
        if (j == 0 && t > 0) ok = ok && mbar_wait_abortable(&bars[D2_EMPTY], (t - 1) & 1, abort_flag);
        const uint32_t s = stage_in();
        if (!ok) return;
        tc_fence_after();
        const uint32_t sB = sW + s * kStage;
        const uint32_t a2 = tmem + kD1Col + (c & 1) * 64;
#pragma unroll
        for (int k = 0; k < 4; ++k)                  // A2 K-step k: half k >> 1, offset 8 (k & 1)
          mma_bf16_ts(tmem + kD2Col, a2 + 32 * (k >> 1) + 8 * (k & 1),
                      desc_sw128(sB + k * 32), kIdesc2, (j > 0 || k > 0) ? 1u : 0u);
        mma_commit(&bars[W_EMPTY0 + s]);
        if (j == kChunks - 1) mma_commit(&bars[D2_FULL]);
        ++k_stage;
      };
      g1(0);
      if (c_total > 1) g1(1);
      for (int c = 0; c < c_total && ok; ++c) {
        g2(c);
        if (c + 2 < c_total) g1(c + 2);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ weight TMA
    // stage order = the MMA issuer's: W1(0) W1(1), then W2(c) W1(c + 2)
    if (lane == 0 && c_total > 0) {
      uint32_t k_stage = 0;
      bool ok = true;
      auto next = [&]() -> uint8_t* {
        const uint32_t s = k_stage % kStages;
        ok = ok && mbar_wait_abortable(&bars[W_EMPTY0 + s], ((k_stage / kStages) & 1) ^ 1, abort_flag);
        mbar_expect_tx(&bars[W_FULL0 + s], kStage);
        return smem + kW + s * kStage;
      };
      auto load_w1 = [&](int c) {                    // hidden rows [64 j, 64 j + 64), K = 256
        uint8_t* dst = next();
        if (!ok) return;
        const int j = c % kChunks;
#pragma unroll
        for (int kb = 0; kb < 4; ++kb)
          bulk_load(dst + kb * 8192, a.w1 + (static_cast<size_t>(kb) * a.HP + 64 * j) * 128, 8192,
                    &bars[W_FULL0 + k_stage % kStages]);
        ++k_stage;
      };
      auto load_w2 = [&](int c) {                    // output rows [0, 256), K = hidden chunk j
        uint8_t* dst = next();
        if (!ok) return;
        const int j = c % kChunks;
        bulk_load(dst, a.w2 + static_cast<size_t>(j) * kCP * 128, kStage,
                  &bars[W_FULL0 + k_stage % kStages]);
        ++k_stage;
      };
      load_w1(0);
      if (c_total > 1) load_w1(1);
      for (int c = 0; c < c_total && ok; ++c) {
        load_w2(c);
        if (c + 2 < c_total) load_w1(c + 2);
      }
    }
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (tid == 0 && *abort_flag) atomicExch(a.status, kStatusTimeout);
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ============================================================== MLP, pipelined
// Warp-specialised persistent version of mlp_kernel for the default width
// (C = 128, H = 256). Roles, per CTA (one CTA per SM):
//   warps 0-3   producer : TMA loads of the three row blocks a tile's conv
//                          reads (rows - d, rows, rows + d), 64-byte channel
//                          boxes into a 2-slot staging ring; conv + LayerNorm
//                          (thread = row); bf16 result written into TMEM
//                          (A operand of GEMM1)
//   warps 4-11  epilogue : GELU of the D1 halves, written back into TMEM as
//                          bf16 (A operand of GEMM2); residual of D2
//   warp 12     MMA      : one elected thread issues all tcgen05.mma
//   warp 13     TMA      : one thread refills staging slots as they are
//                          released, stores finished residual tiles and
//                          loads the next tile's input rows
// H is split in halves (a: h 0..127, b: h 128..255). G1x: D1x = A1 * W1[x]^T,
// G2x: D2 (+)= gelu(D1x) * W2[:, x]^T; both take A from TMEM. MMAs issued by
// one thread execute in order, so G1x(t+1) overwriting D1x cannot overtake
// G2x(t) reading it. After G2a(t) the issuer takes G2b(t) or G1a(t+1),
// whichever is ready first.
// TMEM (512 columns): D1a [0,128) | D1b [128,256) | D2 [256,384) |
// A1[0] [384,448) | A1[1] [448,512). The bf16 GELU output of half x lives in
// D1x's own columns: epilogue warpgroup g packs h [64g, 64g+64) of the half
// into columns [64g, 64g+32), which it has already read.
// Residual (bf16 mode): the tile's input rows arrive by TMA in a 128-byte
// swizzled buffer, the epilogue adds D2 in place, and a TMA tile store
// writes the result: every global access of the tile is a bulk transfer.
// (fp32 mode adds D2 to rows read directly from global memory.)
// Shared memory: W1 64 KB + W2 64 KB (resident), staging 2 slots x 24 KB
// (three row blocks of one 64-byte channel box, 128 rows each), residual
// tile 32 KB, conv weights.
namespace ws {
constexpr int kC = 128, kH = 256, kHalf = 128;
constexpr int kProducerWarps = 4, kEpilogueWarps = 8, kResidualWarps = 4;
constexpr int kResidualWarp0 = kProducerWarps + kEpilogueWarps; // 12
constexpr int kMmaWarp = kResidualWarp0 + kResidualWarps;       // 16
constexpr int kTmaWarp = kMmaWarp + 1;                          // 17
constexpr int kThreads = (kTmaWarp + 1) * 32;                   // 576
constexpr uint32_t kResBox = 128 * 128;                         // 16 KB residual box
constexpr uint32_t kW1 = 0;                                     // 256 x 128 bf16
constexpr uint32_t kW2 = kW1 + kH * kC * 2;                     // 128 x 256 bf16
constexpr uint32_t kStg = kW2 + kC * kH * 2;                    // staging ring
constexpr int kMaxSlots = 5;
enum Bar : int { STG_FULL0 = 0, STG_EMPTY0 = kMaxSlots, A1_FULL0 = 2 * kMaxSlots, A1_FULL1,
                 A1_EMPTY0, A1_EMPTY1, D1A_FULL, D1B_FULL, A2A_FULL, A2B_FULL, D2_FULL,
                 RES_FULL, RES_DONE, D2_EMPTY, W_FULL, kNumBars };
// Staging ring. Split mode (any dilation): a box step covers kBoxBytes of
// channels and a slot holds its three 128-row blocks (rows - d, rows,
// rows + d), 64-byte rows with the 64-byte swizzle. Wide mode (bf16, d <= 64):
// a box step covers 64 channels and a slot holds ONE block of rows
// [t0 - d, t0 + 128 + d) with 128-byte rows and the 128-byte swizzle, which
// contains all three shifted windows: (128 + 2d) row requests per step
// instead of 3 x 128, and a third of the bytes for small d.
template <typename act_t, bool kWide>
struct Layout {
  static constexpr uint32_t kBoxBytes = kWide ? 128 : 64;
  static constexpr int kSlots = 2;
  static constexpr uint32_t kBox = kBoxBytes * 128;               // one 128-row block
  static constexpr uint32_t kSlotBytes = kWide ? 256 * 128 : 3 * kBox;
  static constexpr uint32_t kRes = kStg + kSlots * kSlotBytes;   // 2 boxes (bf16 tile)
  static constexpr uint32_t kConvW = kRes + 2 * kResBox;          // 3 x 128 fp32
  static constexpr uint32_t kBars = kConvW + 3 * kC * 4;
  static constexpr uint32_t kSlot = kBars + kNumBars * 8;
  static constexpr uint32_t kAbort = kSlot + 4;
  static constexpr uint32_t kAlloc = kAbort + 4 + 1024;
  static_assert(kSlots <= kMaxSlots, "staging ring depth");
  static_assert(kAlloc <= 232448, "shared memory per block");
  static_assert(!kWide || sizeof(act_t) == 2, "wide staging is for bf16 activations");
  // 16-byte chunk q of staging row r (swizzle on address bits 7.. of the box)
  __device__ static __forceinline__ uint32_t chunk(int q, int r) {
    return static_cast<uint32_t>(kWide ? (q ^ (r & 7)) : (q ^ ((r >> 1) & 3)));
  }
};
constexpr int kWideMaxDil = 64;
// rows of a wide staging block: 128 + 2d rounded up to whole 8-row swizzle
// atoms (at most 256, the TMA box limit)
__host__ __device__ constexpr int wide_rows(int dil) { return (kTileRows + 2 * dil + 7) & ~7; }
constexpr uint32_t kD2Col = 256, kA1Col = 384;
// TMEM column of the packed bf16 A2 for K-step s (16 h values) of a half
__host__ __device__ constexpr uint32_t a2_col(int s) { return s < 4 ? 8 * s : 64 + 8 * (s - 4); }
}  // namespace ws

struct MlpMaps {
  CUtensorMap stage;   // X_in, staging boxes (Layout::kBoxBytes wide, swizzled)
  CUtensorMap res;     // X_in, 128-byte x 128-row boxes, 128-byte swizzle (bf16 residual)
  CUtensorMap out;     // X_out, same boxes as `res`
};

template <typename act_t, bool kFastGelu, bool kWide>
__global__ void __launch_bounds__(ws::kThreads, 1)
    mlp_ws_kernel(MlpArgs a, const __grid_constant__ MlpMaps maps) {
  using namespace ws;
  using Lay = Layout<act_t, kWide>;
  constexpr uint32_t kBoxBytes = Lay::kBoxBytes, kBox = Lay::kBox, kSlotBytes = Lay::kSlotBytes;
  constexpr uint32_t kRes = Lay::kRes, kConvW = Lay::kConvW, kBars = Lay::kBars;
  constexpr uint32_t kSlot = Lay::kSlot, kAbort = Lay::kAbort;
  constexpr int kSlots = Lay::kSlots;
  constexpr int kCPR = kBoxBytes / 16;                 // 16-byte chunks per staging row
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBars);
  uint32_t* slot = reinterpret_cast<uint32_t*>(smem + kSlot);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kAbort);
  const float* sConvW = reinterpret_cast<const float*>(smem + kConvW);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const act_t* Xi = static_cast<const act_t*>(a.X_in);
  act_t* Xo = static_cast<act_t*>(a.X_out);
  constexpr bool kTmaResidual = sizeof(act_t) == 2;
  constexpr int kBoxCh = kBoxBytes / sizeof(act_t);             // channels per box step
  constexpr int kBoxes = kC / kBoxCh;                           // box steps per tile

  if (warp == kMmaWarp) tmem_alloc(slot, 512);
  if (tid == 0) {
    for (int i = 0; i < kNumBars; ++i) {
      // thread-side barriers count warps (mbar_arrive_warp)
      uint32_t count = 1;
      if ((i >= STG_EMPTY0 && i < STG_EMPTY0 + kMaxSlots) || i == A1_FULL0 || i == A1_FULL1)
        count = kProducerWarps;
      else if (i == A2A_FULL || i == A2B_FULL)
        count = kEpilogueWarps;
      else if (i == RES_DONE || i == D2_EMPTY)
        count = kResidualWarps;
      mbar_init(&bars[i], count);
    }
    *abort_flag = 0;
    mbar_init_fence();
    // W1 and W2 (packed weights only: allowed before griddep_wait) by bulk
    // copies; the MMA warp waits for them
    constexpr uint32_t kWBytes = kH * kC * 2, kPiece = 16384;
    mbar_expect_tx(&bars[W_FULL], 2 * kWBytes);
    for (uint32_t off = 0; off < kWBytes; off += kPiece) {
      bulk_load(smem + kW1 + off, a.w1 + off, kPiece, &bars[W_FULL]);
      bulk_load(smem + kW2 + off, a.w2 + off, kPiece, &bars[W_FULL]);
    }
  }
  {
    if constexpr (sizeof(act_t) == 2) {
      // bf16 activations: conv weights as bf16x2 channel pairs [tap][pair]
      uint32_t* cw = reinterpret_cast<uint32_t*>(smem + kConvW);
      for (int i = tid; i < 3 * kC / 2; i += blockDim.x) {
        const int t = i / (kC / 2), c = 2 * (i % (kC / 2));
        const float v0 = (c < a.C) ? a.convw[t * kC + c] : 0.f;
        const float v1 = (c + 1 < a.C) ? a.convw[t * kC + c + 1] : 0.f;
        cw[i] = pack_bf16x2(v0, v1);
      }
    } else {
      float* cw = reinterpret_cast<float*>(smem + kConvW);
      for (int i = tid; i < 3 * kC; i += blockDim.x) {
        const int c = i % kC;
        cw[i] = (c < a.C) ? a.convw[i] : 0.f;
      }
    }
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  griddep_wait();                          // the previous kernel's outputs are visible
  const uint32_t tmem = *slot;
  const int first = blockIdx.x;
  const int stride = gridDim.x;
  const int n_my = (a.n_tiles > first) ? (a.n_tiles - first + stride - 1) / stride : 0;
  // tiles run from the last example to the first: the statistics kernel just
  // read the last examples (still in L2), and the next one starts at the first
  // examples, which this launch writes last
  auto tile_of = [&](int tit) -> int { return a.n_tiles - 1 - (first + tit * stride); };

  if (warp < kProducerWarps) {
    // ------------------------------------------------------------ producer
    const int quarter = warp & 3;                 // TMEM lane quarter = tile rows
    const int rl = quarter * 32 + lane;           // tile row of this thread
    const uint32_t lane_sel = static_cast<uint32_t>(quarter * 32) << 16;
    uint32_t slotk = 0, phase = 0;   // box step k -> slot k % kSlots, parity (k / kSlots) & 1
    bool ok = true;
    // tiles are per example: tile -> (example n, first position l0); rows
    // outside [0, L) of the example arrive as zero from the 3-D tensor map,
    // which is the conv's zero padding, so no row needs a mask
    float2 st_next = (n_my > 0) ? a.stats[tile_of(0) / a.tpe] : make_float2(0.f, 0.f);
    for (int it = 0; it < n_my && ok; ++it) {
      const int buf = it & 1;
      const float2 st = st_next;                   // statistics loaded one tile ahead
      if (it + 1 < n_my) st_next = a.stats[tile_of(it + 1) / a.tpe];
      const f2 scale2{st.y, st.y};
      const f2 shift2{-st.x * st.y, -st.x * st.y};
      // bf16 fast path: A1 carries a factor 1/2 (exact), which the GELU of
      // D1 / 2 expects (gelu_half_bf16x2)
      constexpr float kA1Scale = (sizeof(act_t) == 2 && kFastGelu) ? 0.5f : 1.0f;
      const uint32_t scale_b = pack_bf16x2(kA1Scale * st.y, kA1Scale * st.y);
      const uint32_t shift_b =
          pack_bf16x2(-kA1Scale * st.x * st.y, -kA1Scale * st.x * st.y);
      for (int b = 0; b < kBoxes; ++b) {
        ok = mbar_wait_abortable(&bars[STG_FULL0 + slotk], phase, abort_flag);
        if (!ok) break;
        if (b == 0) {
          ok = mbar_wait_abortable(&bars[A1_EMPTY0 + buf], ((it >> 1) & 1) ^ 1, abort_flag);
          if (!ok) break;
          tc_fence_after();
        }
        // conv + LayerNorm of this thread's row over the box's channels (the
        // box rows are kBoxBytes wide and swizzled, Layout::chunk)
        const int cbase = b * kBoxCh;              // first channel of the box step
        if constexpr (kWide) {
          // rows rl, rl + d, rl + 2d of the slot's block are this thread's
          // x[l - d], x[l], x[l + d]; two passes of 32 channels
          const uint8_t* blk = smem + kStg + slotk * kSlotBytes;
          const uint32_t* cw2 = reinterpret_cast<const uint32_t*>(smem + kConvW);
          const int rm = rl, rc = rl + a.dil, rp = rl + 2 * a.dil;
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            uint4 sl[4], sc[4], sr[4];
#pragma unroll
            for (int qq = 0; qq < 4; ++qq) {
              const int q = half * 4 + qq;
              sl[qq] = *reinterpret_cast<const uint4*>(blk + rm * 128 + Lay::chunk(q, rm) * 16);
              sc[qq] = *reinterpret_cast<const uint4*>(blk + rc * 128 + Lay::chunk(q, rc) * 16);
              sr[qq] = *reinterpret_cast<const uint4*>(blk + rp * 128 + Lay::chunk(q, rp) * 16);
            }
            if (half == 1) {
              // the step is in registers: release the slot (proxy fence:
              // generic reads before the TMA overwrites it)
              fence_async_smem();
              mbar_arrive_warp(&bars[STG_EMPTY0 + slotk]);
            }
            uint32_t packed[16];
#pragma unroll
            for (int qq = 0; qq < 4; ++qq) {
              const uint4 vl = sl[qq];
              const uint4 vc = sc[qq];
              const uint4 vr = sr[qq];
              const int pr = (cbase + half * 32 + qq * 8) / 2;
              const uint4 w0 = *reinterpret_cast<const uint4*>(cw2 + pr);
              const uint4 w1 = *reinterpret_cast<const uint4*>(cw2 + kC / 2 + pr);
              const uint4 w2 = *reinterpret_cast<const uint4*>(cw2 + kC + pr);
              const uint32_t* pl = &vl.x;
              const uint32_t* pc = &vc.x;
              const uint32_t* pq = &vr.x;
              const uint32_t* p0 = &w0.x;
              const uint32_t* p1 = &w1.x;
              const uint32_t* p2 = &w2.x;
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                uint32_t y = bf2_mul(p2[e], pq[e]);
                y = bf2_fma(p1[e], pc[e], y);
                y = bf2_fma(p0[e], pl[e], y);
                packed[qq * 4 + e] = bf2_fma(y, scale_b, shift_b);
              }
            }
            tmem_st16(tmem + lane_sel + kA1Col + buf * 64 + (cbase + half * 32) / 2, packed);
          }
        } else {
        const uint8_t* bL = smem + kStg + (slotk * 3 + 0) * kBox + rl * kBoxBytes;
        const uint8_t* bC = bL + kBox;
        const uint8_t* bR = bL + 2 * kBox;
        uint32_t packed[kBoxCh / 2];
        if constexpr (sizeof(act_t) == 2) {
          // bf16x2 conv + LayerNorm: y = w0 xl + w1 xc + w2 xr, a = y rstd - mean rstd,
          // four packed operations per channel pair, no unpacking
          const uint32_t* cw2 = reinterpret_cast<const uint32_t*>(smem + kConvW);
          uint4 sl[kCPR], sc[kCPR], sr[kCPR];
#pragma unroll
          for (int q = 0; q < kCPR; ++q) {
            const uint32_t off = Lay::chunk(q, rl) * 16;
            sl[q] = *reinterpret_cast<const uint4*>(bL + off);
            sc[q] = *reinterpret_cast<const uint4*>(bC + off);
            sr[q] = *reinterpret_cast<const uint4*>(bR + off);
          }
          // the row is in registers: release the slot now so its refill
          // overlaps the arithmetic (proxy fence: generic reads before the
          // TMA overwrites the slot)
          fence_async_smem();
          mbar_arrive_warp(&bars[STG_EMPTY0 + slotk]);
#pragma unroll
          for (int q = 0; q < kCPR; ++q) {
            const uint4 vl = sl[q];
            const uint4 vc = sc[q];
            const uint4 vr = sr[q];
            const int pr = (cbase + q * 8) / 2;    // first channel pair of the chunk
            const uint4 w0 = *reinterpret_cast<const uint4*>(cw2 + pr);
            const uint4 w1 = *reinterpret_cast<const uint4*>(cw2 + kC / 2 + pr);
            const uint4 w2 = *reinterpret_cast<const uint4*>(cw2 + kC + pr);
            const uint32_t* pl = &vl.x;
            const uint32_t* pc = &vc.x;
            const uint32_t* pq = &vr.x;
            const uint32_t* p0 = &w0.x;
            const uint32_t* p1 = &w1.x;
            const uint32_t* p2 = &w2.x;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              uint32_t y = bf2_mul(p2[e], pq[e]);
              y = bf2_fma(p1[e], pc[e], y);
              y = bf2_fma(p0[e], pl[e], y);
              packed[q * 4 + e] = bf2_fma(y, scale_b, shift_b);
            }
          }
        } else {
#pragma unroll
        for (int q = 0; q < kCPR; ++q) {           // 16-byte chunks of the row
          const uint32_t off = Lay::chunk(q, rl) * 16;
          const uint4 vl = *reinterpret_cast<const uint4*>(bL + off);
          const uint4 vc = *reinterpret_cast<const uint4*>(bC + off);
          const uint4 vr = *reinterpret_cast<const uint4*>(bR + off);
          constexpr int kE = 16 / sizeof(act_t);  // elements per chunk
          float fl[kE], fc[kE], fr[kE];
          unpack_chunk<act_t>(vl, fl);
          unpack_chunk<act_t>(vc, fc);
          unpack_chunk<act_t>(vr, fr);
          const int c = cbase + q * kE;
#pragma unroll
          for (int e = 0; e < kE; e += 4) {
            const float4 w0 = *reinterpret_cast<const float4*>(sConvW + c + e);
            const float4 w1 = *reinterpret_cast<const float4*>(sConvW + kC + c + e);
            const float4 w2 = *reinterpret_cast<const float4*>(sConvW + 2 * kC + c + e);
            f2 y0 = mul2(f2{w2.x, w2.y}, f2{fr[e], fr[e + 1]});
            f2 y1 = mul2(f2{w2.z, w2.w}, f2{fr[e + 2], fr[e + 3]});
            y0 = fma2(f2{w1.x, w1.y}, f2{fc[e], fc[e + 1]}, y0);
            y1 = fma2(f2{w1.z, w1.w}, f2{fc[e + 2], fc[e + 3]}, y1);
            y0 = fma2(f2{w0.x, w0.y}, f2{fl[e], fl[e + 1]}, y0);
            y1 = fma2(f2{w0.z, w0.w}, f2{fl[e + 2], fl[e + 3]}, y1);
            y0 = fma2(y0, scale2, shift2);
            y1 = fma2(y1, scale2, shift2);
            packed[(q * kE + e) / 2] = pack_bf16x2(y0.x, y0.y);
            packed[(q * kE + e) / 2 + 1] = pack_bf16x2(y1.x, y1.y);
          }
        }
        }
        if constexpr (sizeof(act_t) != 2) {
          // staging consumed: release the slot (the TMA warp refills it with
          // box k + 2). The proxy fence orders these generic-proxy reads
          // before the TMA (async proxy) overwrites the slot; without it the
          // refill can land before the reads complete.
          fence_async_smem();
          mbar_arrive_warp(&bars[STG_EMPTY0 + slotk]);
        }
        // packed channels [cbase, cbase + kBoxCh) -> A1 columns cbase / 2 ...
        const uint32_t col = tmem + lane_sel + kA1Col + buf * 64 + cbase / 2;
        if constexpr (kBoxCh / 2 == 16) {
          tmem_st16(col, packed);
        } else {
          tmem_st8(col, packed);
        }
        }
        if (++slotk == static_cast<uint32_t>(kSlots)) {
          slotk = 0;
          phase ^= 1u;
        }
        if (!ok) break;
      }
      if (!ok) break;
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive_warp(&bars[A1_FULL0 + buf]);
    }
  } else if (warp < kResidualWarp0) {
    // ------------------------------------------------------------ GELU epilogue
    const int ew = warp - kProducerWarps;          // 0..7
    const int quarter = warp & 3;                  // TMEM lane quarter of this warp
    const int g = ew >> 2;                         // warpgroup: half columns [64g, 64g+64)
    const uint32_t lane_sel = static_cast<uint32_t>(quarter * 32) << 16;   // rows of this warp
    for (int it = 0; it < n_my; ++it) {
      bool ok = true;
#pragma unroll 1
      for (int hh = 0; hh < 2; ++hh) {
        // GELU of half hh, in place: D1x fp32 -> packed bf16 A2x
        ok = mbar_wait_abortable(&bars[hh ? D1B_FULL : D1A_FULL], it & 1, abort_flag);
        if (!ok) break;
        tc_fence_after();
        const uint32_t base = tmem + lane_sel + hh * kHalf + g * 64;
#pragma unroll 1
        for (int j = 0; j < 2; ++j) {
          uint32_t r[32];
          tmem_ld32(base + j * 32, r);
          uint32_t p[16];
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            if constexpr (kFastGelu && sizeof(act_t) == 2) {
              p[q] = gelu_half_bf16x2(__uint_as_float(r[2 * q]), __uint_as_float(r[2 * q + 1]));
            } else if constexpr (kFastGelu) {
              p[q] = gelu_bf16x2(__uint_as_float(r[2 * q]), __uint_as_float(r[2 * q + 1]));
            } else {
              p[q] = pack_bf16x2(gelu_tanh<false>(__uint_as_float(r[2 * q])),
                                 gelu_tanh<false>(__uint_as_float(r[2 * q + 1])));
            }
          }
          tmem_st16(base + j * 16, p);
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive_warp(&bars[hh ? A2B_FULL : A2A_FULL]);
      }
      if (!ok) break;
    }
  } else if (warp < kMmaWarp) {
    // ------------------------------------------------------------ residual epilogue
    // X_out = X_in + D2 for whole rows (thread = row, all channels); D2 is
    // released (D2_EMPTY) as soon as it has been read, before the tile store
    const int quarter = warp & 3;
    const int rl = quarter * 32 + lane;
    const uint32_t lane_sel = static_cast<uint32_t>(quarter * 32) << 16;
    uint8_t* sRes = smem + kRes;
    for (int it = 0; it < n_my; ++it) {
      if constexpr (kTmaResidual) {
        // residual of D2 through the TMA-loaded input tile, in place
        // the tile's input rows arrive by TMA (issued by this group's leader
        // after the previous tile's store left the buffer)
        const bool leader = (warp == kResidualWarp0 && lane == 0);
        auto load_res = [&](int tit) {
          const int tile = tile_of(tit);
          const int n = tile / a.tpe, l0 = (tile - n * a.tpe) * kTileRows;
          mbar_expect_tx(&bars[RES_FULL], 2 * kResBox);
          tma_load_3d(sRes, &maps.res, 0, l0, n, &bars[RES_FULL]);
          tma_load_3d(sRes + kResBox, &maps.res, 64, l0, n, &bars[RES_FULL]);
        };
        if (it == 0 && leader) load_res(0);
        if (!mbar_wait_abortable(&bars[RES_FULL], it & 1, abort_flag)) break;
        if (!mbar_wait_abortable(&bars[D2_FULL], it & 1, abort_flag)) break;
        tc_fence_after();
#pragma unroll 1
        for (int jj = 0; jj < 4; ++jj) {
          const int g = jj >> 1, j = jj & 1;
          uint8_t* rowp = sRes + g * kResBox + rl * 128;   // channels [64g, 64g + 64)
          uint4 x[4];
#pragma unroll
          for (int q = 0; q < 4; ++q)                     // 8 channels per chunk
            x[q] = *reinterpret_cast<const uint4*>(rowp + (((j * 4 + q) ^ (rl & 7)) * 16));
          uint32_t d[32];
          tmem_ld32(tmem + lane_sel + kD2Col + jj * 32, d);
          if (jj == 3) {
            tc_fence_before();
            mbar_arrive_warp(&bars[D2_EMPTY]);            // D2 fully read
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t* dq = d + q * 8;
            // x + bf16(D2) in bf16x2 (one extra rounding of the update)
            *reinterpret_cast<uint4*>(rowp + (((j * 4 + q) ^ (rl & 7)) * 16)) = make_uint4(
                bf2_add(x[q].x, pack_bf16x2(__uint_as_float(dq[0]), __uint_as_float(dq[1]))),
                bf2_add(x[q].y, pack_bf16x2(__uint_as_float(dq[2]), __uint_as_float(dq[3]))),
                bf2_add(x[q].z, pack_bf16x2(__uint_as_float(dq[4]), __uint_as_float(dq[5]))),
                bf2_add(x[q].w, pack_bf16x2(__uint_as_float(dq[6]), __uint_as_float(dq[7]))));
          }
        }
        fence_async_smem();                               // generic writes -> TMA store
        mbar_arrive_warp(&bars[RES_DONE]);
        if (leader) {
          if (!mbar_wait_abortable(&bars[RES_DONE], it & 1, abort_flag)) break;
          const int tile = tile_of(it);
          const int n = tile / a.tpe, l0 = (tile - n * a.tpe) * kTileRows;
          tma_store_3d(&maps.out, sRes, 0, l0, n);        // rows past L are clipped
          tma_store_3d(&maps.out, sRes + kResBox, 64, l0, n);
          bulk_commit();
          if (it + 1 < n_my) {
            bulk_wait_read0();                            // the tile buffer is free again
            load_res(it + 1);
          } else {
            bulk_wait0();                                 // stores complete before exit
          }
        }
      } else {
        // residual of D2 on rows read directly from global memory (fp32)
        const int tile = tile_of(it);
        const int n = tile / a.tpe, l = (tile - n * a.tpe) * kTileRows + rl;
        const bool rv = l < a.L;
        const long long r = (long long)n * a.L + l;
        constexpr int kVE = 16 / sizeof(act_t);
        constexpr int kPre = 32 / kVE;
        if (!mbar_wait_abortable(&bars[D2_FULL], it & 1, abort_flag)) break;
        tc_fence_after();
#pragma unroll 1
        for (int g = 0; g < 2; ++g) {
        const act_t* xrow = Xi + r * kC + g * 64;
        act_t* orow = Xo + r * kC + g * 64;
        uint4 xin[kPre];
#pragma unroll
        for (int q = 0; q < kPre; ++q)
          xin[q] = rv ? *reinterpret_cast<const uint4*>(xrow + q * kVE) : make_uint4(0, 0, 0, 0);
#pragma unroll 1
        for (int j = 0; j < 2; ++j) {
          uint32_t d[32];
          tmem_ld32(tmem + lane_sel + kD2Col + g * 64 + j * 32, d);
          if (j == 1) {
#pragma unroll
            for (int q = 0; q < kPre; ++q)
              xin[q] = rv ? *reinterpret_cast<const uint4*>(xrow + 32 + q * kVE)
                          : make_uint4(0, 0, 0, 0);
          }
          if (rv) {
#pragma unroll
            for (int q = 0; q < kPre; ++q)
              *reinterpret_cast<uint4*>(orow + j * 32 + q * kVE) =
                  add_residual<act_t>(xin[q], d + q * kVE);
          }
        }
        }
        tc_fence_before();
        mbar_arrive_warp(&bars[D2_EMPTY]);
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    // (the weights' bulk copies are waited for even without tiles, so no
    // copy into this CTA's shared memory outlives it)
    bool w_ok = true;
    if (lane == 0) w_ok = mbar_wait_abortable(&bars[W_FULL], 0, abort_flag);
    if (lane == 0 && n_my > 0 && w_ok) {
      const uint32_t sW1 = smem_u32(smem + kW1), sW2 = smem_u32(smem + kW2);
      constexpr uint32_t kIdesc = idesc_bf16(kTileRows, 128);
      auto g1 = [&](int hh, int buf) {  // D1x = A1(tmem) * W1[hh*128 : hh*128+128]^T, K = 128
        const uint32_t d = tmem + hh * kHalf;
#pragma unroll
        for (int kk = 0; kk < kC / 16; ++kk) {
          const uint64_t db =
              desc_sw128(sW1 + (kk >> 2) * (kH * 128) + hh * (kHalf * 128) + (kk & 3) * 32);
          mma_bf16_ts(d, tmem + kA1Col + buf * 64 + 8 * kk, db, kIdesc, kk > 0 ? 1u : 0u);
        }
      };
      auto g2 = [&](int hh) {  // D2 (+)= A2x(tmem) * W2[:, x]^T, K = 128
        const uint32_t d = tmem + kD2Col;
#pragma unroll
        for (int kk = 0; kk < kHalf / 16; ++kk) {
          const uint64_t db =
              desc_sw128(sW2 + (hh * 2 + (kk >> 2)) * (kC * 128) + (kk & 3) * 32);
          mma_bf16_ts(d, tmem + hh * kHalf + a2_col(kk), db, kIdesc,
                      (hh > 0 || kk > 0) ? 1u : 0u);
        }
      };
      bool ok = mbar_wait_abortable(&bars[A1_FULL0], 0, abort_flag);
      if (ok) {
        tc_fence_after();
        g1(0, 0);
        mma_commit(&bars[D1A_FULL]);
        g1(1, 0);
        mma_commit(&bars[D1B_FULL]);
        mma_commit(&bars[A1_EMPTY0]);
      }
      for (int it = 0; ok && it < n_my; ++it) {
        const bool next = it + 1 < n_my;
        const int nbuf = (it + 1) & 1;
        ok = mbar_wait_abortable(&bars[A2A_FULL], it & 1, abort_flag);
        if (ok && it > 0) ok = mbar_wait_abortable(&bars[D2_EMPTY], (it - 1) & 1, abort_flag);
        if (!ok) break;
        tc_fence_after();
        g2(0);
        // G2b(t) and G1a(t+1), whichever is ready first
        bool g2b_done = false, g1a_done = !next;
        const uint32_t a2b = smem_u32(&bars[A2B_FULL]);
        const uint32_t a1f = smem_u32(&bars[A1_FULL0 + nbuf]);
        const uint64_t t0 = global_ns();
        for (uint32_t spin = 0; !(g2b_done && g1a_done); ++spin) {
          if (!g2b_done && mbar_try(a2b, it & 1)) {
            tc_fence_after();
            g2(1);
            mma_commit(&bars[D2_FULL]);
            g2b_done = true;
            continue;
          }
          if (!g1a_done && mbar_try(a1f, ((it + 1) >> 1) & 1)) {
            tc_fence_after();
            g1(0, nbuf);
            mma_commit(&bars[D1A_FULL]);
            g1a_done = true;
            continue;
          }
          if ((spin & 255u) == 255u && (*abort_flag || global_ns() - t0 > kWaitNs)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
        }
        if (!ok) break;
        if (next) {
          g1(1, nbuf);
          mma_commit(&bars[D1B_FULL]);
          mma_commit(&bars[A1_EMPTY0 + nbuf]);
        }
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ TMA warp
    if (lane == 0 && n_my > 0) {
      // staging box step k -> (tile k / kBoxes, box k % kBoxes) into slot k % kSlots
      auto issue = [&](uint32_t k, uint32_t slotk) {
        const int tit = static_cast<int>(k / kBoxes);
        const int b = static_cast<int>(k % kBoxes);
        const int tile = tile_of(tit);
        const int n = tile / a.tpe, l0 = (tile - n * a.tpe) * kTileRows;
        if constexpr (kWide) {
          // one block of rows [l0 - d, l0 - d + wide_rows(d)) (the map's box)
          mbar_expect_tx(&bars[STG_FULL0 + slotk], wide_rows(a.dil) * kBoxBytes);
          tma_load_3d(smem + kStg + slotk * kSlotBytes, &maps.stage, b * kBoxCh, l0 - a.dil, n,
                      &bars[STG_FULL0 + slotk]);
        } else {
          mbar_expect_tx(&bars[STG_FULL0 + slotk], kSlotBytes);
#pragma unroll
          for (int blk = 0; blk < 3; ++blk)
            tma_load_3d(smem + kStg + (slotk * 3 + blk) * kBox, &maps.stage, b * kBoxCh,
                        l0 + (blk - 1) * a.dil, n, &bars[STG_FULL0 + slotk]);
        }
      };
      const uint32_t n_steps = static_cast<uint32_t>(n_my) * kBoxes;
      uint32_t k_next = 0;
      for (; k_next < n_steps && k_next < static_cast<uint32_t>(kSlots); ++k_next)
        issue(k_next, k_next);
      uint32_t eslot = 0, ephase = 0;      // slot / parity of the next refill's STG_EMPTY
      const uint64_t t0 = global_ns();
      uint64_t last_progress = t0;
      for (uint32_t spin = 0; k_next < n_steps; ++spin) {
        if (mbar_try(smem_u32(&bars[STG_EMPTY0 + eslot]), ephase)) {
          issue(k_next, eslot);
          ++k_next;
          if (++eslot == static_cast<uint32_t>(kSlots)) {
            eslot = 0;
            ephase ^= 1u;
          }
          last_progress = global_ns();
        } else if ((spin & 255u) == 255u) {
          if (*abort_flag || global_ns() - last_progress > kWaitNs) {
            *abort_flag = 1;
            break;
          }
        }
      }
    }
    __syncwarp();
  }
  // drain: every MMA this CTA issued has been waited on by the residual
  // warps (D2_FULL of the last tile) unless the pipeline aborted.
  tc_fence_before();
  __syncthreads();
  if (tid == 0 && *abort_flag) atomicExch(a.status, kStatusTimeout);
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ============================================================== heads
// Profile head: P[b, o, j] = bias[o] + sum_{c < Cin, t < 75} F[o, c, t]
//   * Xc[b, c, T + j + t - 37],  j in [0, Lout)
// where Xc = concat(X, X_ctl) along channels, zero outside [0, L)
// (upstream cherimoya.py:182-184, 379-384). A block handles kHeadJ output
// positions of one example; the input window is staged channel-major in
// shared memory. Warp w sums channels c = w, w + 4, ...; lane i produces
// kHeadPer consecutive positions with a sliding register window; the four
// warp partials are added in a fixed order.
constexpr int kHeadJ = 128;
constexpr int kHeadPer = 4;
constexpr int kHeadWarps = 4;
constexpr int kHeadWin = kHeadJ + kHeadTaps - 1;   // 202

template <typename act_t>
__global__ void __launch_bounds__(kHeadWarps * 32) profile_head_kernel(
    const act_t* __restrict__ X, const float* __restrict__ X_ctl, const float* __restrict__ F,
    const float* __restrict__ fbias, float* __restrict__ profile, int L, int C, int CP,
    int n_ctl, int n_out, int T, int Lout) {
  extern __shared__ float win[];   // [Cin][kHeadWin], then [kHeadWarps][kHeadJ]
  const int b = blockIdx.y;
  const int j0 = blockIdx.x * kHeadJ;
  const int Cin = C + n_ctl;
  float* part = win + Cin * kHeadWin;
  const int p0 = T + j0 - kHeadPad;     // sequence position of win[.][0]
  for (int idx = threadIdx.x; idx < kHeadWin * Cin; idx += blockDim.x) {
    const int w = idx / Cin, c = idx - (idx / Cin) * Cin;
    const int p = p0 + w;
    float v = 0.f;
    if (p >= 0 && p < L) {
      v = (c < C) ? to_f32<act_t>(X[((long long)b * L + p) * CP + c])
                  : X_ctl[((long long)b * n_ctl + (c - C)) * L + p];
    }
    win[c * kHeadWin + w] = v;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int jl = lane * kHeadPer;
  for (int o = 0; o < n_out; ++o) {
    float acc[kHeadPer];
#pragma unroll
    for (int e = 0; e < kHeadPer; ++e) acc[e] = 0.f;
    const float* Fo = F + (long long)o * Cin * kHeadTaps;
    for (int c = warp; c < Cin; c += kHeadWarps) {
      const float* wrow = win + c * kHeadWin + jl;
      const float* frow = Fo + c * kHeadTaps;
      float sw[kHeadPer];
#pragma unroll
      for (int e = 0; e < kHeadPer - 1; ++e) sw[e + 1] = wrow[e];
#pragma unroll 5
      for (int t = 0; t < kHeadTaps; ++t) {
#pragma unroll
        for (int e = 0; e < kHeadPer - 1; ++e) sw[e] = sw[e + 1];
        sw[kHeadPer - 1] = wrow[t + kHeadPer - 1];
        const float f = __ldg(frow + t);
#pragma unroll
        for (int e = 0; e < kHeadPer; ++e) acc[e] = fmaf(f, sw[e], acc[e]);
      }
    }
#pragma unroll
    for (int e = 0; e < kHeadPer; ++e) part[warp * kHeadJ + jl + e] = acc[e];
    __syncthreads();
    if (warp == 0) {
      const float bo = fbias[o];
#pragma unroll
      for (int e = 0; e < kHeadPer; ++e) {
        const int j = j0 + jl + e;
        float v = part[jl + e];
#pragma unroll
        for (int w = 1; w < kHeadWarps; ++w) v += part[w * kHeadJ + jl + e];
        if (j < Lout) profile[((long long)b * n_out + o) * Lout + j] = v + bo;
      }
    }
    __syncthreads();
  }
}

// Count head: logcount[b, g] = bias[g] + sum_c Wl[g, c] mean_{l in [T, L-T)} X[b, l, c]
//   (+ Wl[g, C] * log(1 + sum_{k, l in [T, L-T)} X_ctl[b, k, l]) with controls)
// (upstream cherimoya.py:185-186, 387-399). One block per example, one
// thread per channel.
template <typename act_t>
__global__ void __launch_bounds__(256) count_head_kernel(
    const act_t* __restrict__ X, const float* __restrict__ X_ctl, const float* __restrict__ Wl,
    const float* __restrict__ lbias, float* __restrict__ logcounts, int L, int C, int CP,
    int n_ctl, int n_groups, int T) {
  __shared__ float mean_s[256];
  __shared__ float ctl_s;
  __shared__ float red[8];
  const int b = blockIdx.x;
  const int c = threadIdx.x;
  const int Lout = L - 2 * T;
  if (c < C) {
    float s = 0.f;
    const act_t* Xb = X + ((long long)b * L + T) * CP + c;
    for (int l = 0; l < Lout; ++l) s += to_f32<act_t>(Xb[(long long)l * CP]);
    mean_s[c] = s / static_cast<float>(Lout);
  }
  if (threadIdx.x == 0) {
    float cs = 0.f;
    for (int k = 0; k < n_ctl; ++k) {
      const float* xc = X_ctl + ((long long)b * n_ctl + k) * L + T;
      for (int l = 0; l < Lout; ++l) cs += xc[l];
    }
    ctl_s = logf(cs + 1.0f);
  }
  __syncthreads();
  const int Cin = C + (n_ctl > 0 ? 1 : 0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int g = 0; g < n_groups; ++g) {
    float v = 0.f;
    if (c < C) v = Wl[(long long)g * Cin + c] * mean_s[c];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = lbias[g];
      for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += red[i];
      if (n_ctl > 0) t += Wl[(long long)g * Cin + C] * ctl_s;
      logcounts[(long long)b * n_groups + g] = t;
    }
    __syncthreads();
  }
}

// ============================================================== heads, tcgen05
// Profile head as a GEMM plus a diagonal reduction (upstream
// cherimoya.py:182-184, 379-384):
//   Z[w, t] = sum_c Xc[p0 + w, c] * F[o, c, t]        (tcgen05, fp32 in TMEM)
//   P[o, j] = bias[o] + sum_{t < 75} Z[j + t, t]       (fixed-order sums)
// over the window w in [0, Lout + 74) starting at sequence position
// p0 = T - 37, for one (output channel o, example b) per CTA. F is packed
// transposed (taps x channels, K-major) as bf16 hi + lo parts, so X * F is
// carried to ~16 bits; in fp32 mode X is split the same way (3 MMAs). The
// count head is fused: the example's o == 0 CTA accumulates per-channel
// sums of the rows in [T, L - T) while it stages them (fixed order), then
// logcount[g] = bias[g] + sum_c Wl[g, c] mean[c] (+ Wl[g, C] log(1 + sum ctl)).
namespace hd {
constexpr int kNP = 80;            // 75 taps padded to an MMA N
constexpr int kZStride = 77;       // Z ring row stride (floats): conflict-free diagonals
constexpr int kRing = 208;         // ring rows: one tile + the 74-row halo, rounded up
constexpr int kThreads = 128;

// sum over u < n of ring[((row0 + u) mod kRing) * kZStride + t0 + u], in order
// of u (row0 < kRing): consecutive taps of one output are one ring row and one
// column apart, a stride of kZStride + 1 floats, with at most one wrap of the
// ring in between
__device__ __forceinline__ float ring_diag_sum(const float* ring, int row0, int t0, int n) {
  const int n1 = min(n, kRing - row0);
  const float* p = ring + row0 * kZStride + t0;
  float acc = 0.f;
#pragma unroll 4
  for (int u = 0; u < n1; ++u) acc += p[u * (kZStride + 1)];
  const float* q = ring + t0 + n1;
#pragma unroll 4
  for (int u = 0; u < n - n1; ++u) acc += q[u * (kZStride + 1)];
  return acc;
}
}  // namespace hd

struct HeadArgs {
  int* status;            // set on a timed-out wait
  const void* X;          // (B * L, CP) act_t
  const float* X_ctl;     // (B, n_ctl, L) or null
  const uint8_t* fb;      // packed F: per output o, [hi | lo] each kNP x CPH bf16 swizzled
  const float* fbias;     // (n_out)
  const float* lw;        // (n_groups, C (+1))
  const float* lbias;     // (n_groups)
  float* profile;         // (B, n_out, Lout)
  float* logcounts;       // (B, n_groups)
  int L, C, CP, CPH, n_ctl, n_out, n_groups, T, Lout;
  int batch;              // head_fused_kernel: examples
};

__host__ __device__ constexpr uint32_t head_smem_bytes(int CPH, int a_splits) {
  return static_cast<uint32_t>(2 * hd::kNP * CPH * 2 + a_splits * kTileRows * CPH * 2 +
                               hd::kRing * hd::kZStride * 4 + 2048 + 64 + 1024);
}

template <typename act_t, int kASplits>
__global__ void __launch_bounds__(hd::kThreads) head_kernel(HeadArgs a) {
  using namespace hd;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int CPH = a.CPH;
  uint8_t* sB = smem;                                          // [2][kNP x CPH]
  uint8_t* sA = sB + 2 * kNP * CPH * 2;                        // [kASplits][128 x CPH]
  float* ring = reinterpret_cast<float*>(sA + kASplits * kTileRows * CPH * 2);
  float* red = ring + kRing * kZStride;                        // 512 floats
  uint64_t* bar = reinterpret_cast<uint64_t*>(red + 512);
  uint32_t* slot = reinterpret_cast<uint32_t*>(bar + 1);
  const int o = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool counts = (o == 0);

  if (warp == 0) tmem_alloc(slot, 128);
  if (tid == 0) {
    mbar_init(bar, 1);
    mbar_init_fence();
  }
  {  // this output's packed F (hi and lo)
    const uint4* g = reinterpret_cast<const uint4*>(a.fb + (size_t)o * 2 * kNP * CPH * 2);
    uint4* d = reinterpret_cast<uint4*>(sB);
    for (int i = tid; i < 2 * kNP * CPH * 2 / 16; i += blockDim.x) d[i] = g[i];
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *slot;
  const int W = a.Lout + kHeadTaps - 1;
  const int n_tiles = (W + kTileRows - 1) / kTileRows;
  const int p0 = a.T - kHeadPad;
  const int chunks = CPH / 8;                   // 16-byte channel chunks per row
  const int my_chunk = tid % chunks;
  const int row_step = kHeadThreadsRows(chunks);
  float csum[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) csum[e] = 0.f;
  float ctl_sum = 0.f;
  const act_t* Xb = static_cast<const act_t*>(a.X) + (long long)b * a.L * a.CP;
  const uint32_t sA_addr = smem_u32(sA), sB_addr = smem_u32(sB);
  const uint32_t idesc = idesc_bf16(kTileRows, kNP);
  bool ok = true;

  for (int k = 0; k < n_tiles; ++k) {
    // ---- stage window rows [128k, 128k + 128) as bf16 (hi [, lo]) operand tiles
    for (int rr = tid / chunks; rr < kTileRows; rr += row_step) {
      const int w = k * kTileRows + rr;
      const int p = p0 + w;
      const int c = my_chunk * 8;
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = 0.f;
      if (w < W && p >= 0 && p < a.L) {
        if (c + 8 <= a.C) {
          load8(Xb + (long long)p * a.CP + c, v);
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int ce = c + e;
            if (ce < a.C) v[e] = to_f32<act_t>(Xb[(long long)p * a.CP + ce]);
            else if (ce < a.C + a.n_ctl)
              v[e] = a.X_ctl[((long long)b * a.n_ctl + (ce - a.C)) * a.L + p];
          }
        }
        if (counts && p >= a.T && p < a.L - a.T) {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            if (c + e < a.C) csum[e] += v[e];
            else if (c + e < a.C + a.n_ctl) ctl_sum += v[e];
          }
        }
      }
      uint32_t hi[4], lo[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        hi[e] = pack_bf16x2(v[2 * e], v[2 * e + 1]);
        if (kASplits > 1) {
          const float h0 = __uint_as_float(hi[e] << 16), h1 = __uint_as_float(hi[e] & 0xFFFF0000u);
          lo[e] = pack_bf16x2(v[2 * e] - h0, v[2 * e + 1] - h1);
        }
      }
      const uint32_t off = sw128_offset(rr, c, kTileRows);
      *reinterpret_cast<uint4*>(sA + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
      if (kASplits > 1)
        *reinterpret_cast<uint4*>(sA + kTileRows * CPH * 2 + off) =
            make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    // ---- Z = A_hi F_hi + A_hi F_lo (+ A_lo F_hi)
    if (tid == 0) {
      tc_fence_after();
      const int ksteps = CPH / 16;
      uint32_t acc = 0;
      for (int term = 0; term < (kASplits > 1 ? 3 : 2); ++term) {
        const int ai = (term == 2) ? 1 : 0;
        const int bi = (term == 1) ? 1 : 0;
        for (int kk = 0; kk < ksteps; ++kk) {
          const uint64_t da = desc_sw128(sA_addr + ai * (kTileRows * CPH * 2) +
                                         (kk >> 2) * (kTileRows * 128) + (kk & 3) * 32);
          const uint64_t db = desc_sw128(sB_addr + bi * (kNP * CPH * 2) +
                                         (kk >> 2) * (kNP * 128) + (kk & 3) * 32);
          mma_bf16(tmem, da, db, idesc, acc);
          acc = 1;
        }
      }
      mma_commit(bar);
    }
    ok = mbar_wait(bar, k & 1);
    if (__syncthreads_or(!ok)) {
      if (tid == 0) atomicExch(a.status, kStatusTimeout);
      break;
    }
    tc_fence_after();
    // ---- Z tile -> ring rows (128k + row) mod kRing (columns 0..74)
    {
      const int rr = warp * 32 + lane;
      float* zrow = ring + ((k * kTileRows + rr) % kRing) * kZStride;
      const uint32_t lane_sel = static_cast<uint32_t>(warp * 32) << 16;
#pragma unroll 1
      for (int part = 0; part < 3; ++part) {
        const int col = part == 0 ? 0 : (part == 1 ? 32 : 48);   // 48..79 overlaps 32..63
        uint32_t r[32];
        tmem_ld32(tmem + lane_sel + col, r);
        tmem_ld_wait();
#pragma unroll
        for (int q = 0; q < 32; ++q) {
          const int t = col + q;
          if ((part < 2 || t >= 64) && t < kHeadTaps) zrow[t] = __uint_as_float(r[q]);
        }
      }
    }
    tc_fence_before();
    __syncthreads();
    // ---- outputs whose 75 rows are now all in the ring
    // rows j .. j + 74 of output j lie in tiles <= k and the ring still holds
    // rows >= 128k - 80
    const int j_lo = (k == 0) ? 0 : k * kTileRows - (kHeadTaps - 1);
    const int j_hi = (k == n_tiles - 1) ? a.Lout
                                        : min(a.Lout, k * kTileRows + kTileRows - (kHeadTaps - 1));
    for (int j = j_lo + tid; j < j_hi; j += blockDim.x) {
      const float acc = ring_diag_sum(ring, j % kRing, 0, kHeadTaps);
      a.profile[((long long)b * a.n_out + o) * a.Lout + j] = acc + a.fbias[o];
    }
    __syncthreads();
  }
  if (counts) {
    // fixed-order reduction of the per-thread channel sums
    for (int e = 0; e < 8; ++e) {
      red[tid] = csum[e];
      __syncthreads();
      if (tid < chunks) {
        const int c = tid * 8 + e;
        float s = 0.f;
        for (int i = tid; i < blockDim.x; i += chunks) s += red[i];
        if (c < a.C) red[256 + c] = s / static_cast<float>(a.Lout);
      }
      __syncthreads();
    }
    red[tid] = ctl_sum;
    __syncthreads();
    if (tid == 0) {
      float cs = 0.f;
      for (int i = 0; i < blockDim.x; ++i) cs += red[i];
      red[255] = logf(cs + 1.0f);
    }
    __syncthreads();
    const int cin = a.C + (a.n_ctl > 0 ? 1 : 0);
    for (int g = warp; g < a.n_groups; g += blockDim.x / 32) {
      float v = 0.f;
      for (int c = lane; c < a.C; c += 32) v += a.lw[(long long)g * cin + c] * red[256 + c];
#pragma unroll
      for (int sh = 16; sh > 0; sh >>= 1) v += __shfl_xor_sync(0xffffffffu, v, sh);
      if (lane == 0) {
        float t = a.lbias[g] + v;
        if (a.n_ctl > 0) t += a.lw[(long long)g * cin + a.C] * red[255];
        a.logcounts[(long long)b * a.n_groups + g] = t;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
}

// Profile + count head for bf16 activations without control tracks (C <= 128):
// persistent, one CTA per SM looping over (output, example) work items. The
// window tiles come straight from HBM by TMA (3-D tensor map, 128-byte
// swizzle: two boxes of 64 channels = the K-major operand layout the MMA
// reads), three tiles in flight; rows outside [0, L) arrive as zero, the
// profile conv's padding. Z = X F^T goes to one of two TMEM buffers. The
// count head rides in the same MMA: the five spare operand rows after the 75
// taps hold the count Linear's weights (output 0 only), so Z[w, 75 + g] =
// sum_c X[w, c] lw[g, c] and logcount[g] = lbias[g] + sum_w Z[w, 75 + g] / Lout
// over the trimmed window.
// Warp 17 streams the window tiles (three buffers, each refilled as soon as
// the MMAs that read it have completed); warp 16 issues the MMAs. With F as
// hi + lo (C = 128) the two halves are stacked into one N = 160 operand (rows
// 80.. = lo), so each window tile is read once per K step and Z = Z_hi + Z_lo
// is added in the epilogue. Z of tile g goes to TMEM buffer
// g & 1 and is taken by epilogue group g & 1 (warps 0-7, 8-15), so the two
// groups work on consecutive tiles at the same time. A group copies its Z tile
// to its own shared-memory buffer and sums the tile's part of every diagonal
// it touches: outputs j = 128 k - 74 + s, s < 202, each over its taps t with
// row j + t inside the tile, in four 20-tap items combined by shuffles in a
// fixed order. Outputs 128 k .. 128 k + 53 are complete in the tile. The 74
// outputs that continue into the next tile (s >= 128) go, with the running
// sums of the count columns, to the group's carry buffer, and the next tile's
// group adds its own part to them. The carry is handed over tile by tile
// (c_full / c_empty), so every output and count is summed in tile order
// (deterministic).
namespace hd3 {
constexpr int kGroupWarps = 8;                           // epilogue warps per group
constexpr int kGroupThreads = kGroupWarps * 32;
constexpr int kEpiThreads = 2 * kGroupThreads;           // two groups, alternate tiles
constexpr int kIssuerWarp = kEpiThreads / 32;           // MMAs
constexpr int kTmaWarp = kIssuerWarp + 1;                // window-tile loads
constexpr int kThreads = kEpiThreads + 64;
constexpr int kABufs = 3;
constexpr int kMaxGroups = hd::kNP - kHeadTaps;          // 5 spare operand rows
constexpr int kZCols = 2 * hd::kNP;                      // TMEM columns per Z buffer
constexpr int kCarry = kHeadTaps - 1;                    // outputs that straddle two tiles
constexpr int kSpan = kTileRows + kCarry;                // outputs a tile contributes to
constexpr int kPartTaps = 20;                            // taps per partial-sum item
constexpr int kParts = 4;                                // items per output (75 taps)
static_assert(kParts * kPartTaps >= kHeadTaps && (kParts - 1) * kPartTaps < kHeadTaps,
              "tap parts");
constexpr int kPasses = (kSpan * kParts + kGroupThreads - 1) / kGroupThreads;
constexpr uint32_t kBox = 128 * 128;                     // 16 KB: 64 channels x 128 rows
constexpr uint32_t kB = 0;                               // F hi | lo: 2 x 80 x 128 bf16
constexpr uint32_t kA = 40960;                           // kABufs x 2 boxes
constexpr uint32_t kZsBytes = kTileRows * hd::kZStride * 4;
constexpr uint32_t kZs = kA + kABufs * 2 * kBox;         // [group][128 rows][kZStride] fp32
constexpr int kCarryStride = 80;                         // tail partials, then count sums
constexpr uint32_t kCarryOff = kZs + 2 * kZsBytes;       // [group][kCarryStride] fp32
constexpr uint32_t kRed = kCarryOff + 2 * kCarryStride * 4;   // [group][4 warps][kMaxGroups]
constexpr uint32_t kBars = kRed + 2 * 4 * kMaxGroups * 4;
// a_full[3] z_full[2] z_free[2] mma_done a_free[3] c_full[2] c_empty[2] f_full
constexpr int kNumBars = 2 * kABufs + 10;
constexpr uint32_t kSlot = kBars + kNumBars * 8;
constexpr uint32_t kAlloc = kSlot + 16 + 1024;
static_assert(kA % 1024 == 0 && 2 * hd::kNP * 128 * 2 <= kA, "operand layout");
static_assert(kBars % 8 == 0 && kCarry + kMaxGroups <= kCarryStride, "carry layout");
static_assert(kAlloc <= 232448, "shared memory per block");
}  // namespace hd3

// CPH = 128: F as bf16 hi + lo (two MMA terms); CPH = 256: each window tile
// arrives in two 128-channel halves that accumulate into the same Z, and F is
// bf16 (the precision of the upstream bf16 autocast path for this conv), so
// the shared-memory layout is the same for both widths.
template <int CPH>
__global__ void __launch_bounds__(hd3::kThreads, 1) head_fused_kernel(
    HeadArgs a, const __grid_constant__ CUtensorMap tmap) {
  using namespace hd;
  using hd3::kBox;
  static_assert(CPH == 128 || CPH == 256, "head width");
  constexpr int kSub = CPH / 128;                       // 128-channel halves per tile
  constexpr int kTerms = CPH == 128 ? 2 : 1;            // F hi (+ lo)
  static_assert(kTerms * kNP * CPH * 2 <= hd3::kA, "operand F");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sB = smem + hd3::kB;
  uint8_t* sA = smem + hd3::kA;
  uint64_t* a_full = reinterpret_cast<uint64_t*>(smem + hd3::kBars);   // [kABufs]
  uint64_t* z_full = a_full + hd3::kABufs;                              // [2]
  uint32_t* slot = reinterpret_cast<uint32_t*>(smem + hd3::kSlot);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int W = a.Lout + kHeadTaps - 1;                 // window rows per example
  const int n_tiles = (W + kTileRows - 1) / kTileRows;
  const int p0 = a.T - kHeadPad;                        // first window position
  const int n_items = a.n_out * a.batch;
  const int n_mine = (n_items > (int)blockIdx.x)
                         ? (n_items - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x
                         : 0;
  const int total = n_mine * n_tiles;                   // this CTA's tile sequence

  uint64_t* z_free = z_full + 2;                                        // [2]
  uint64_t* mma_done = z_free + 2;
  uint64_t* a_free = mma_done + 1;                                      // [kABufs]
  uint64_t* c_full = a_free + hd3::kABufs;                              // [2]
  uint64_t* c_empty = c_full + 2;                                       // [2]
  uint64_t* f_full = c_empty + 2;
  if (warp == 0) tmem_alloc(slot, 512);
  if (tid == 0) {
    for (int i = 0; i < hd3::kNumBars; ++i) mbar_init(&a_full[i], 1);
    for (int e = 0; e < 2; ++e) {                       // one arrive per group warp
      mbar_init(&z_free[e], hd3::kGroupWarps);
      mbar_init(&c_full[e], hd3::kGroupWarps);
      mbar_init(&c_empty[e], hd3::kGroupWarps);
    }
    mbar_init_fence();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  griddep_wait();                          // the previous kernel's outputs are visible
  const uint32_t tmem = *slot;
  // Position of this CTA's sub-steps (item = blockIdx.x + i * gridDim.x,
  // tile k of it, channel half sub), advanced one step at a time so that a
  // step costs no integer division (only a change of item does).
  struct Cursor {
    int sub, k, item, o, b;
  };
  auto cur_init = [&](Cursor& c) {
    c.sub = 0;
    c.k = 0;
    c.item = static_cast<int>(blockIdx.x);
    c.o = c.item / a.batch;
    c.b = c.item - c.o * a.batch;
  };
  auto cur_next = [&](Cursor& c, int subs) {
    if (++c.sub < subs) return;
    c.sub = 0;
    if (++c.k < n_tiles) return;
    c.k = 0;
    c.item += static_cast<int>(gridDim.x);
    c.o = c.item / a.batch;
    c.b = c.item - c.o * a.batch;
  };
  bool ok = true;
  if (warp == hd3::kTmaWarp) {
    // ------------------------------------------------------------ window tiles
    // sub-step gs = (tile g, channel half gs % kSub) -> A buffer gs % kABufs,
    // refilled once the MMAs of sub-step gs - kABufs have completed
    if (lane == 0) {
      const int total_sub = total * kSub;
      Cursor lc;
      cur_init(lc);
      for (int gs = 0; gs < total_sub && ok; ++gs, cur_next(lc, kSub)) {
        const int buf = gs % hd3::kABufs;
        if (gs >= hd3::kABufs)
          ok = mbar_wait(&a_free[buf], ((gs - hd3::kABufs) / hd3::kABufs) & 1);
        if (!ok) break;
        const int x0 = 128 * lc.sub;
        mbar_expect_tx(&a_full[buf], 2 * kBox);
        tma_load_3d(sA + buf * 2 * kBox, &tmap, x0, p0 + lc.k * kTileRows, lc.b, &a_full[buf]);
        tma_load_3d(sA + buf * 2 * kBox + kBox, &tmap, x0 + 64, p0 + lc.k * kTileRows, lc.b,
                    &a_full[buf]);
      }
    }
    __syncwarp();
  } else if (warp == hd3::kIssuerWarp) {
    // ------------------------------------------------------------ MMAs
    const uint32_t sA_addr = smem_u32(sA), sB_addr = smem_u32(sB);
    constexpr uint32_t kSlabB = kTerms * kNP * 128;      // bytes per 64-channel slab of F
    const uint32_t idesc = idesc_bf16(kTileRows, kTerms * kNP);
    int cur_o = -1;
    uint32_t done_phase = 0, f_phase = 0;
    Cursor ic;
    cur_init(ic);
    for (int g = 0; g < total && ok; ++g, cur_next(ic, 1)) {
      const int o = ic.o;
      if (o != cur_o) {
        // operand F of output o by bulk copies, once the MMAs reading the
        // previous one have completed: per 64-channel slab, the hi rows then
        // (C = 128) the lo rows
        if (lane == 0) {
          if (g > 0) {
            mma_commit(mma_done);
            ok = mbar_wait(mma_done, done_phase & 1);
          }
          if (ok) {
            constexpr uint32_t kSlabBytes = kNP * 128;   // one slab of one term
            constexpr uint32_t kTermBytes = kSlabBytes * (CPH / 64);
            const uint8_t* src = a.fb + (size_t)o * 2 * kNP * CPH * 2;
            mbar_expect_tx(f_full, kTerms * kTermBytes);
            for (int term = 0; term < kTerms; ++term)
              for (int slab = 0; slab < CPH / 64; ++slab)
                bulk_load(sB + (slab * kTerms + term) * kSlabBytes,
                          src + term * kTermBytes + slab * kSlabBytes, kSlabBytes, f_full);
            ok = mbar_wait(f_full, f_phase & 1);
          }
        }
        if (g > 0) ++done_phase;
        ++f_phase;
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
        cur_o = o;
      }
      if (lane == 0) {
        const int zb = g & 1;
        for (int half = 0; half < kSub && ok; ++half) {
          const int gs = g * kSub + half, buf = gs % hd3::kABufs;
          ok = mbar_wait(&a_full[buf], (gs / hd3::kABufs) & 1);
          // TMEM buffer zb was released by the epilogue of tile g - 2
          if (half == 0) ok = ok && mbar_wait(&z_free[zb], ((g >> 1) & 1) ^ 1);
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t da = desc_sw128(sA_addr + buf * 2 * kBox + (kk >> 2) * kBox +
                                           (kk & 3) * 32);
            const uint64_t db = desc_sw128(sB_addr + (2 * half + (kk >> 2)) * kSlabB +
                                           (kk & 3) * 32);
            mma_bf16(tmem + zb * hd3::kZCols, da, db, idesc, (half > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(&a_free[buf]);
          if (half == kSub - 1) mma_commit(&z_full[zb]);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    }
  } else {
    // ------------------------------------------------------------ epilogue
    using hd3::kCarry;
    using hd3::kMaxGroups;
    const int e = warp / hd3::kGroupWarps;              // group: tiles g with g & 1 == e
    const int gw = warp % hd3::kGroupWarps;
    const int rq = gw & 3;                              // TMEM lane quarter (warp % 4)
    const int ch = gw >> 2;                             // column half: [0, 48) / [48, 80)
    const int gt = tid % hd3::kGroupThreads;
    const uint32_t lane_sel = static_cast<uint32_t>(rq * 32) << 16;
    const uint32_t zcol = tmem + e * hd3::kZCols;
    // Z column c = hi column c (+ lo column kNP + c); count columns likewise
    auto zload16 = [&](int c0, uint32_t (&r)[16]) {
      tmem_ld16(zcol + lane_sel + c0, r);
      if (kTerms == 2) {
        uint32_t q2[16];
        tmem_ld16(zcol + lane_sel + kNP + c0, q2);
#pragma unroll
        for (int q = 0; q < 16; ++q)
          r[q] = __float_as_uint(__uint_as_float(r[q]) + __uint_as_float(q2[q]));
      }
    };
    const int w = rq * 32 + lane;                       // tile row = TMEM lane
    float* Zs = reinterpret_cast<float*>(smem + hd3::kZs + e * hd3::kZsBytes);
    float* carry_mine = reinterpret_cast<float*>(smem + hd3::kCarryOff) + e * hd3::kCarryStride;
    const float* carry_prev =
        reinterpret_cast<const float*>(smem + hd3::kCarryOff) + (e ^ 1) * hd3::kCarryStride;
    float* red = reinterpret_cast<float*>(smem + hd3::kRed) + e * 4 * kMaxGroups;
    Cursor ec;
    cur_init(ec);
    if (e == 1) cur_next(ec, 1);
    int fb_o = -1;
    float fbias = 0.f;                                  // bias of output fb_o
    for (int g = e, n = 0; g < total; g += 2, ++n, cur_next(ec, 1), cur_next(ec, 1)) {
      const int b = ec.b, o = ec.o, k = ec.k;
      if (o != fb_o) {
        fbias = __ldg(&a.fbias[o]);
        fb_o = o;
      }
      const bool counts = (o == 0);
      ok = mbar_wait(&z_full[e], n & 1);
      if (!ok) break;
      tc_fence_after();
      // ---- Z tile -> Zs (rows w, taps); count columns summed per warp
      {
        float* zrow = Zs + w * kZStride;
        if (ch == 0) {
#pragma unroll 1
          for (int c0 = 0; c0 < 48; c0 += 16) {
            uint32_t r[16];
            zload16(c0, r);
#pragma unroll
            for (int q = 0; q < 16; ++q) zrow[c0 + q] = __uint_as_float(r[q]);
          }
          tc_fence_before();
          mbar_arrive_warp(&z_free[e]);                 // TMEM buffer e is free again
        } else {
          uint32_t r[16];
          zload16(48, r);
#pragma unroll
          for (int q = 0; q < 16; ++q) zrow[48 + q] = __uint_as_float(r[q]);
          uint32_t r2[16];
          zload16(64, r2);                              // taps 64..74, count columns
#pragma unroll
          for (int q = 0; q < kHeadTaps - 64; ++q) zrow[64 + q] = __uint_as_float(r2[q]);
          tc_fence_before();
          mbar_arrive_warp(&z_free[e]);
          if (counts) {
            const int wr = k * kTileRows + w;           // window row
            const bool in = wr >= kHeadPad && wr < kHeadPad + a.Lout;
#pragma unroll
            for (int gi = 0; gi < kMaxGroups; ++gi) {
              float v = in ? __uint_as_float(r2[kHeadTaps - 64 + gi]) : 0.f;
#pragma unroll
              for (int sh = 16; sh > 0; sh >>= 1) v += __shfl_xor_sync(0xffffffffu, v, sh);
              if (lane == 0) red[rq * kMaxGroups + gi] = v;
            }
          }
        }
      }
      named_sync(1 + e, hd3::kGroupThreads);
      // ---- this tile's part of the diagonals: item = 4 s + p covers taps
      // [20 p, 20 p + 20) of output s whose rows s - 74 + t lie in [0, 128)
      // (the four passes' chains run interleaved, each summed in tap order)
      float pv[hd3::kPasses];
      int pidx[hd3::kPasses], plen[hd3::kPasses];
#pragma unroll
      for (int pass = 0; pass < hd3::kPasses; ++pass) {
        const int item = pass * hd3::kGroupThreads + gt;
        const int so = item >> 2, pp = item & 3;
        const int t_lo = max(pp * hd3::kPartTaps, kCarry - so);
        const int t_hi = min(min(pp * hd3::kPartTaps + hd3::kPartTaps, kHeadTaps), hd3::kSpan - so);
        plen[pass] = (so < hd3::kSpan) ? max(0, t_hi - t_lo) : 0;
        pidx[pass] = (so - kCarry + t_lo) * kZStride + t_lo;
        pv[pass] = 0.f;
      }
#pragma unroll 4
      for (int u = 0; u < hd3::kPartTaps; ++u) {
#pragma unroll
        for (int pass = 0; pass < hd3::kPasses; ++pass)
          if (u < plen[pass]) pv[pass] += Zs[pidx[pass] + u * (kZStride + 1)];
      }
#pragma unroll
      for (int pass = 0; pass < hd3::kPasses; ++pass) {
        float v = pv[pass];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        pv[pass] = v;                                   // (p0 + p1) + (p2 + p3)
      }
      float tile_cnt = 0.f;                             // threads gt < kMaxGroups
      if (counts && gt < kMaxGroups)
        tile_cnt = ((red[gt] + red[kMaxGroups + gt]) + red[2 * kMaxGroups + gt]) +
                   red[3 * kMaxGroups + gt];
      // ---- outputs: s < 74 complete with the previous tile's carry, 74 <= s
      // < 128 are complete here
      if (g > 0) {
        ok = mbar_wait(&c_full[e ^ 1], ((g - 1) >> 1) & 1);
        if (!ok) break;
      }
      float* prof = a.profile + ((long long)b * a.n_out + o) * a.Lout;
#pragma unroll
      for (int pass = 0; pass < 2; ++pass) {
        const int so = (pass * hd3::kGroupThreads + gt) >> 2;
        const int j = k * kTileRows - kCarry + so;
        if ((gt & 3) == 0 && j < a.Lout) {
          if (so < kCarry) {
            if (k > 0) prof[j] = (carry_prev[so] + pv[pass]) + fbias;
          } else {
            prof[j] = pv[pass] + fbias;
          }
        }
      }
      float run = 0.f;                                  // count sums through tile k
      if (counts && gt < kMaxGroups) {
        run = (k == 0) ? tile_cnt : carry_prev[kCarry + gt] + tile_cnt;
        if (k == n_tiles - 1 && gt < a.n_groups)
          a.logcounts[(long long)b * a.n_groups + gt] = a.lbias[gt] + run / static_cast<float>(a.Lout);
      }
      if (g > 0) mbar_arrive_warp(&c_empty[e ^ 1]);     // done with the previous carry
      // ---- carry for the next tile: outputs s >= 128, running count sums
      if (n > 0) {
        ok = mbar_wait(&c_empty[e], (n - 1) & 1);
        if (!ok) break;
      }
#pragma unroll
      for (int pass = 2; pass < hd3::kPasses; ++pass) {
        const int so = (pass * hd3::kGroupThreads + gt) >> 2;
        if ((gt & 3) == 0 && so < hd3::kSpan) carry_mine[so - kTileRows] = pv[pass];
      }
      if (gt < kMaxGroups) carry_mine[kCarry + gt] = run;
      mbar_arrive_warp(&c_full[e]);
      named_sync(1 + e, hd3::kGroupThreads);            // Zs and red are free again
    }
  }
  if (!ok) atomicExch(a.status, kStatusTimeout);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ============================================================== wait self-test
// The bounded-wait path of every pipeline, exercised on purpose: thread 0
// waits, with the pipelines' own abortable wait (2 s of wall time), on an
// mbarrier that nothing arrives on, then records the timeout in the status
// word as a stalled pipeline would. Nothing is in flight when it returns, so
// the context stays usable.
__global__ void wait_timeout_selftest_kernel(int* status) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    mbar_init_fence();
  }
  __syncthreads();
  if (threadIdx.x == 0 && !mbar_wait_abortable(&bar, 0, &abort_flag))
    atomicExch(status, kStatusTimeout);
}

// ============================================================== scoring
// Row-wise softmax of a reference profile flattened over (n_out, Lout), and
// (pw != nullptr) the row's ProfileWrapper value
//   sum_i softmax(x)_i (x_i - mean(x)) = sum_i softmax(x)_i x_i - mean(x)
// (upstream wrappers.py:71-99: mean-centred flattened logits weighted by
// their softmax, which the centring does not change).
__global__ void __launch_bounds__(256) softmax_rows_kernel(const float* __restrict__ logits,
                                                           float* __restrict__ probs, int len,
                                                           float* __restrict__ pw) {
  __shared__ float red[8];
  __shared__ float bcast;
  const long long base = (long long)blockIdx.x * len;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float m = -INFINITY;
  for (int i = threadIdx.x; i < len; i += blockDim.x) m = fmaxf(m, logits[base + i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = red[0];
    for (int i = 1; i < 8; ++i) t = fmaxf(t, red[i]);
    bcast = t;
  }
  __syncthreads();
  m = bcast;
  float s = 0.f;
  for (int i = threadIdx.x; i < len; i += blockDim.x) s += expf(logits[base + i] - m);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  __syncthreads();
  if (lane == 0) red[warp] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < 8; ++i) t += red[i];
    bcast = t;
  }
  __syncthreads();
  const float inv = 1.0f / bcast;
  float sx = 0.f, spx = 0.f;
  for (int i = threadIdx.x; i < len; i += blockDim.x) {
    const float x = logits[base + i];
    const float p = expf(x - m) * inv;
    probs[base + i] = p;
    sx += x;
    spx = fmaf(p, x, spx);
  }
  if (pw == nullptr) return;
  __shared__ float red2[2][8];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sx += __shfl_xor_sync(0xffffffffu, sx, o);
    spx += __shfl_xor_sync(0xffffffffu, spx, o);
  }
  if (lane == 0) {
    red2[0][warp] = sx;
    red2[1][warp] = spx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float tx = 0.f, tp = 0.f;
    for (int i = 0; i < 8; ++i) {
      tx += red2[0][i];
      tp += red2[1][i];
    }
    pw[blockIdx.x] = tp - tx / static_cast<float>(len);
  }
}

// ExpectedCountsWrapper (upstream wrappers.py:125-166): for example n and
// signal group g (channels [off[g], off[g + 1]) of the profile), a joint softmax
// over the group's channels and positions times expm1(logcount[n, g]).
constexpr int kMaxEpilogueGroups = 64;
struct GroupOffsets {
  int off[kMaxEpilogueGroups + 1];
};
__global__ void __launch_bounds__(256) expected_counts_kernel(
    const float* __restrict__ profile, const float* __restrict__ logcounts, int n_out, int Lout,
    int n_groups, GroupOffsets go, float* __restrict__ out) {
  __shared__ float red[8];
  __shared__ float bcast;
  const int g = blockIdx.x, n = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long base = ((long long)n * n_out + go.off[g]) * Lout;
  const int len = (go.off[g + 1] - go.off[g]) * Lout;
  float m = -INFINITY;
  for (int i = threadIdx.x; i < len; i += blockDim.x) m = fmaxf(m, profile[base + i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = red[0];
    for (int i = 1; i < 8; ++i) t = fmaxf(t, red[i]);
    bcast = t;
  }
  __syncthreads();
  m = bcast;
  float s = 0.f;
  for (int i = threadIdx.x; i < len; i += blockDim.x) s += expf(profile[base + i] - m);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  __syncthreads();
  if (lane == 0) red[warp] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < 8; ++i) t += red[i];
    bcast = t;
  }
  __syncthreads();
  const float scale = expm1f(logcounts[(long long)n * n_groups + g]) / bcast;
  for (int i = threadIdx.x; i < len; i += blockDim.x)
    out[base + i] = expf(profile[base + i] - m) * scale;
}

// Jensen-Shannon distance between softmax(logits[i]) and probs[ref_of(i)]
// over `len` values (upstream performance.py:138-207: zero-probability
// terms contribute 0, natural log), plus the log-count delta of every
// group. ref_of(i) = i / per_ref for ISM passes (i counted from mut0), or
// i for variant pairs (per_ref = 1).
__device__ __forceinline__ float kl_term(float p, float q) {
  return (p != 0.f && q != 0.f) ? p * logf(p / q) : 0.f;
}

struct ScoreArgs {
  const float* logits;      // (n, len) mutant / alt profiles
  const float* ref_probs;   // (n_ref, len)
  const float* lc;          // (n, n_groups) mutant / alt logcounts
  const float* lc_ref;      // (n_ref, n_groups)
  int len;
  int n_groups;
  long long mut0;           // global index of row 0 (ISM)
  int per_ref;              // rows per reference (ISM: 3 * width; variants: 1)
  int ism;                  // 1: ISM output layout, 0: variant layout
  int ism_start, ism_width; // ISM: window
  const int8_t* bases;      // ISM: reference bases (n_ref, L)
  int L;
  float* d_logcount;        // ISM: (n_ref, n_groups, 4, W); variant: (n, n_groups)
  float* jsd;               // ISM: (n_ref, 4, W); variant: (n)
  const float* pw_ref;      // ISM, optional: ProfileWrapper value of each reference
  float* d_pw;              // ISM, optional: (n_ref, 4, W) its change in the mutant
};

__global__ void __launch_bounds__(256) score_kernel(ScoreArgs a) {
  __shared__ float red[8];
  __shared__ float bcast;
  const int row = blockIdx.x;
  const long long gm = a.mut0 + row;
  const int ref = static_cast<int>(gm / a.per_ref);
  const float* x = a.logits + (long long)row * a.len;
  const float* q = a.ref_probs + (long long)ref * a.len;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float m = -INFINITY;
  for (int i = threadIdx.x; i < a.len; i += blockDim.x) m = fmaxf(m, x[i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = red[0];
    for (int i = 1; i < 8; ++i) t = fmaxf(t, red[i]);
    bcast = t;
  }
  __syncthreads();
  m = bcast;
  float s = 0.f;
  for (int i = threadIdx.x; i < a.len; i += blockDim.x) s += expf(x[i] - m);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  __syncthreads();
  if (lane == 0) red[warp] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < 8; ++i) t += red[i];
    bcast = t;
  }
  __syncthreads();
  const float inv = 1.0f / bcast;
  // JSD terms, and for the ProfileWrapper value sum(x) and sum(softmax * x)
  float j = 0.f, sx = 0.f, spx = 0.f;
  for (int i = threadIdx.x; i < a.len; i += blockDim.x) {
    const float p1 = expf(x[i] - m) * inv;
    const float p2 = q[i];
    const float mid = 0.5f * (p1 + p2);
    j += kl_term(p1, mid) + kl_term(p2, mid);
    sx += x[i];
    spx = fmaf(p1, x[i], spx);
  }
  __shared__ float red3[3][8];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    j += __shfl_xor_sync(0xffffffffu, j, o);
    sx += __shfl_xor_sync(0xffffffffu, sx, o);
    spx += __shfl_xor_sync(0xffffffffu, spx, o);
  }
  if (lane == 0) {
    red3[0][warp] = j;
    red3[1][warp] = sx;
    red3[2][warp] = spx;
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  float jt = 0.f, tx = 0.f, tp = 0.f;
  for (int i = 0; i < 8; ++i) {
    jt += red3[0][i];
    tx += red3[1][i];
    tp += red3[2][i];
  }
  jt *= 0.5f;
  if (a.ism) {
    const int rem = static_cast<int>(gm - (long long)ref * a.per_ref);
    const int w = rem / 3, k = rem - 3 * (rem / 3);
    const int p = a.ism_start + w;
    const int alt = ((a.bases[(long long)ref * a.L + p] & 3) + 1 + k) & 3;
    a.jsd[((long long)ref * 4 + alt) * a.ism_width + w] = jt;
    if (a.d_pw)
      a.d_pw[((long long)ref * 4 + alt) * a.ism_width + w] =
          (tp - tx / static_cast<float>(a.len)) - a.pw_ref[ref];
    for (int g = 0; g < a.n_groups; ++g) {
      const float d = a.lc[(long long)row * a.n_groups + g] - a.lc_ref[(long long)ref * a.n_groups + g];
      a.d_logcount[(((long long)ref * a.n_groups + g) * 4 + alt) * a.ism_width + w] = d;
    }
  } else {
    a.jsd[gm] = jt;
    for (int g = 0; g < a.n_groups; ++g)
      a.d_logcount[gm * a.n_groups + g] =
          a.lc[(long long)row * a.n_groups + g] - a.lc_ref[(long long)ref * a.n_groups + g];
  }
}

// ISM entries whose base equals the reference base: the mutant is the
// reference, both scores are 0.
__global__ void ism_fill_ref_kernel(const int8_t* __restrict__ bases, int L, int start, int W,
                                    int n_groups, int n_ref, float* d_logcount, float* jsd,
                                    float* d_pw) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)n_ref * W) return;
  const int n = static_cast<int>(i / W), w = static_cast<int>(i - (long long)n * W);
  const int b = bases[(long long)n * L + start + w] & 3;
  jsd[((long long)n * 4 + b) * W + w] = 0.f;
  if (d_pw) d_pw[((long long)n * 4 + b) * W + w] = 0.f;
  for (int g = 0; g < n_groups; ++g)
    d_logcount[(((long long)n * n_groups + g) * 4 + b) * W + w] = 0.f;
}

// ============================================================== packing
// fp32 (R, K) row-major source -> bf16 K-major 128B-swizzled tile of RP x KP
// (zero padded), values multiplied by `scale`.
__global__ void pack_sw128_kernel(const float* __restrict__ src, int R, int K, int RP, int KP,
                                  float scale, uint8_t* __restrict__ dst) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= RP * KP) return;
  const int r = i / KP, k = i - (i / KP) * KP;
  const float v = (r < R && k < K) ? src[(long long)r * K + k] * scale : 0.f;
  *reinterpret_cast<__nv_bfloat16*>(dst + sw128_offset(r, k, RP)) = __float2bfloat16_rn(v);
}

// hi / lo split of an fp32 (R, K) matrix into two bf16 swizzled tiles
// (lo = value - bf16(value)); dst holds [hi | lo], each RP x KP.
// taps > 0: src rows are (channels x taps) channel-major and the packed K
// order is tap-major, k = channels * t + c  <-  src column taps * c + t.
// extra (optional, length R) fills column K: the stem bias, multiplied by a
// constant-one A column in the bf16 stem and by a zero column elsewhere.
__global__ void pack_sw128_split_kernel(const float* __restrict__ src, int R, int K, int RP,
                                        int KP, int taps, const float* __restrict__ extra,
                                        uint8_t* __restrict__ dst) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= RP * KP) return;
  const int r = i / KP, k = i - (i / KP) * KP;
  int ks = k;
  if (taps > 0 && k < K) {
    const int chans = K / taps;
    ks = (k % chans) * taps + k / chans;
  }
  float v = (r < R && k < K) ? src[(long long)r * K + ks] : 0.f;
  if (extra != nullptr && k == K && r < R) v = extra[r];
  const __nv_bfloat16 h = __float2bfloat16_rn(v);
  const uint32_t off = sw128_offset(r, k, RP);
  *reinterpret_cast<__nv_bfloat16*>(dst + off) = h;
  *reinterpret_cast<__nv_bfloat16*>(dst + (size_t)RP * KP * 2 + off) =
      __float2bfloat16_rn(v - __bfloat162float(h));
}

// Profile-head weight F (n_out, Cin, 75) -> per output o a transposed
// [taps x channels] operand, hi and lo: dst[o] = [hi | lo], each NP x CPH.
// When lw is given (no control tracks, n_groups <= NP - taps), the spare rows
// taps .. taps + n_groups - 1 of output 0 hold the count Linear's weights
// lw[g, c], so the same MMA produces sum_c X[w, c] lw[g, c].
__global__ void pack_head_kernel(const float* __restrict__ F, int n_out, int Cin, int taps,
                                 int NP, int CPH, const float* __restrict__ lw, int n_groups,
                                 uint8_t* __restrict__ dst) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)n_out * NP * CPH) return;
  const int o = static_cast<int>(i / ((long long)NP * CPH));
  const int rem = static_cast<int>(i - (long long)o * NP * CPH);
  const int t = rem / CPH, c = rem - (rem / CPH) * CPH;
  float v = (t < taps && c < Cin) ? F[((long long)o * Cin + c) * taps + t] : 0.f;
  if (lw != nullptr && o == 0 && t >= taps && t - taps < n_groups && c < Cin)
    v = lw[(long long)(t - taps) * Cin + c];
  const __nv_bfloat16 h = __float2bfloat16_rn(v);
  uint8_t* base = dst + (size_t)o * 2 * NP * CPH * 2;
  const uint32_t off = sw128_offset(t, c, NP);
  *reinterpret_cast<__nv_bfloat16*>(base + off) = h;
  *reinterpret_cast<__nv_bfloat16*>(base + (size_t)NP * CPH * 2 + off) =
      __float2bfloat16_rn(v - __bfloat162float(h));
}

// fp32 (3, C) -> (3, CP) zero padded.
__global__ void pack_convw_kernel(const float* __restrict__ src, int C, int CP,
                                  float* __restrict__ dst) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= 3 * CP) return;
  const int t = i / CP, c = i - (i / CP) * CP;
  dst[i] = (c < C) ? src[t * C + c] : 0.f;
}

// (rows, C) <-> (rows, CP) channel padding of activations.
template <typename act_t>
__global__ void pad_channels_kernel(const act_t* __restrict__ src, act_t* __restrict__ dst,
                                    long long rows, int C, int CP) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * CP) return;
  const long long r = i / CP;
  const int c = static_cast<int>(i - r * CP);
  dst[i] = (c < C) ? src[r * C + c] : from_f32<act_t>(0.f);
}
template <typename act_t>
__global__ void unpad_channels_kernel(const act_t* __restrict__ src, act_t* __restrict__ dst,
                                      long long rows, int C, int CP) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * C) return;
  const long long r = i / C;
  const int c = static_cast<int>(i - r * C);
  dst[i] = src[r * CP + c];
}

__global__ void copy_f32_kernel(const float* __restrict__ src, float* __restrict__ dst, long long n) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[i] = src[i];
}

}  // namespace chm
