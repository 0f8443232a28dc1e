// chm_engine.cu -- C ABI of the Cherimoya B200 engine (see
// include/cherimoya_b200.h). Host orchestration only: validation, workspace
// carving, kernel dispatch. No entry point allocates device memory.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <type_traits>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "../../include/cherimoya_b200.h"
#include "chm_kernels.cuh"

using namespace chm;

namespace {

thread_local long long g_launches = 0;

// ---- optional per-launch CUDA-event timing (benchmark instrumentation)
enum KClass { kKStem = 0, kKStats = 1, kKMlp = 2, kKProfile = 3, kKCount = 4, kKScore = 5,
              kKOther = 6, kKClasses = 7 };
struct TimedLaunch {
  int cls;
  cudaEvent_t start, stop;
};
struct Timing {
  bool enabled = false;
  std::vector<TimedLaunch> pending;
  std::vector<cudaEvent_t> pool;
  cudaEvent_t get() {
    if (!pool.empty()) {
      cudaEvent_t e = pool.back();
      pool.pop_back();
      return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
  }
};
thread_local Timing g_timing;

// RAII bracket around one kernel launch.
struct LaunchTimer {
  TimedLaunch t{};
  cudaStream_t st;
  bool on;
  LaunchTimer(int cls, cudaStream_t s) : st(s), on(g_timing.enabled) {
    if (!on) return;
    t.cls = cls;
    t.start = g_timing.get();
    t.stop = g_timing.get();
    cudaEventRecord(t.start, st);
  }
  ~LaunchTimer() {
    if (!on) return;
    cudaEventRecord(t.stop, st);
    g_timing.pending.push_back(t);
  }
};

constexpr size_t kAlign = 1024;
size_t align_up(size_t v, size_t a = kAlign) { return (v + a - 1) / a * a; }
int round64(int v) { return (v + 63) / 64 * 64; }
// padded channel width: 64, 128 or 256 (kernels tile channels in 64-wide
// operand boxes and assume the width divides their thread layouts)
int pad_channels(int c) { return c <= 64 ? 64 : (c <= 128 ? 128 : round64(c) <= 256 ? 256 : round64(c)); }

struct Dims {
  int C, CP, H, HP, L, T, Lout, n_layers, n_out, n_groups, n_ctl, mode;
  float rs;
  int act_bytes() const { return mode == CHM_MODE_BF16 ? 2 : 4; }
};

Dims dims_of(const chm_model_desc* d) {
  Dims m;
  m.C = d->n_filters;
  m.CP = pad_channels(d->n_filters);
  m.H = d->expansion * d->n_filters;
  m.HP = round64(m.H);
  m.L = d->seq_len;
  m.T = d->trimming;
  m.Lout = d->seq_len - 2 * d->trimming;
  m.n_layers = d->n_layers;
  m.n_out = d->n_outputs;
  m.n_groups = d->n_groups;
  m.n_ctl = d->n_control_tracks;
  m.mode = d->mode;
  m.rs = d->residual_scale;
  return m;
}

// ---- packed weight buffer layout
struct PackLayout {
  size_t stem_w, stem_b, stem_pk, layers, layer_stride, l_convw, l_w1, l_w2;
  size_t head_f, head_fb, head_lw, head_lb, head_pk, total;
};

// channel width of the head's GEMM operand (a divisor-friendly padding)
int head_cph(const Dims& m) {
  const int cin = m.C + m.n_ctl;
  return cin <= 64 ? 64 : (cin <= 128 ? 128 : 256);
}

PackLayout pack_layout(const Dims& m) {
  PackLayout p;
  size_t o = 0;
  p.stem_w = o; o = align_up(o + (size_t)m.C * 4 * kStemTaps * 4);
  p.stem_b = o; o = align_up(o + (size_t)m.C * 4);
  p.stem_pk = o; o = align_up(o + 2 * (size_t)m.CP * sm::kK * 2);
  p.l_convw = 0;
  p.l_w1 = align_up(3 * (size_t)m.CP * 4);
  p.l_w2 = align_up(p.l_w1 + (size_t)m.HP * m.CP * 2);
  p.layer_stride = align_up(p.l_w2 + (size_t)m.CP * m.HP * 2);
  p.layers = o; o += p.layer_stride * m.n_layers;
  const size_t cin = (size_t)m.C + m.n_ctl;
  p.head_f = o; o = align_up(o + (size_t)m.n_out * cin * kHeadTaps * 4);
  p.head_fb = o; o = align_up(o + (size_t)m.n_out * 4);
  p.head_lw = o; o = align_up(o + (size_t)m.n_groups * (m.C + (m.n_ctl > 0 ? 1 : 0)) * 4);
  p.head_lb = o; o = align_up(o + (size_t)m.n_groups * 4);
  p.head_pk = o; o = align_up(o + (size_t)m.n_out * 2 * hd::kNP * head_cph(m) * 2);
  p.total = o;
  return p;
}

// ---- forward workspace layout (for `batch` rows)
struct FwdLayout {
  size_t status, stats, xa, xb, total;
};

FwdLayout fwd_layout(const Dims& m, int batch) {
  FwdLayout f;
  size_t o = 0;
  f.status = o; o = align_up(o + 256);
  f.stats = o; o = align_up(o + (size_t)batch * 8);
  const size_t act = (size_t)batch * m.L * m.CP * m.act_bytes();
  f.xa = o; o = align_up(o + act);
  f.xb = o; o = align_up(o + act);
  f.total = o;
  return f;
}

int device_sms() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
  return sms > 0 ? sms : 148;
}

// Launch `k`; with `pdl` under programmatic stream serialization, so the grid
// may start while the stream's previous kernel finishes. Such a kernel calls
// griddep_wait() before it touches anything an earlier kernel of the stream
// wrote; before that it reads only packed weights. The first kernel of every
// C-ABI call is launched without it, so weight packing that precedes a call
// has completed before any of the call's kernels reads the weights.
template <typename... KArgs, typename... Args>
void launch_k(bool pdl, void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem,
              cudaStream_t st, Args... args) {
  if (!pdl) {
    k<<<grid, block, smem, st>>>(args...);
    return;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, k, args...);
}


int launch_status() {
  ++g_launches;
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    fprintf(stderr, "cherimoya_b200: launch failed: %s\n", cudaGetErrorString(e));
    return CHM_ERR_LAUNCH;
  }
  return CHM_OK;
}

#define CHM_TRY(expr)              \
  do {                             \
    const int _s = (expr);         \
    if (_s != CHM_OK) return _s;   \
  } while (0)

// ---- TMA tensor maps (driver entry point resolved through the runtime, so
// the library does not link libcuda directly)
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}


// Activations as a 3-D tensor (channels, L, batch) of 128-byte x 128-row x 1
// boxes with the 128-byte swizzle: rows outside [0, L) of an example read as
// zero (the conv's zero padding).
int make_act_tmap3(CUtensorMap* map, const void* base, int batch, int L, int CP) {
  EncodeTiledFn fn = encode_tiled();
  if (!fn) return CHM_ERR_CUDA;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return CHM_ERR_WORKSPACE;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(CP), static_cast<cuuint64_t>(L),
                              static_cast<cuuint64_t>(batch)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(CP) * 2,
                                 static_cast<cuuint64_t>(CP) * 2 * L};
  const cuuint32_t box[3] = {64u, 128u, 1u};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? CHM_OK : CHM_ERR_CUDA;
}

// Activations as a 3-D tensor (channels, L, batch) with boxes of box_bytes of
// channels x box_rows positions x 1 example, swizzle = box width (32, 64 or
// 128 bytes); positions outside [0, L) read as zero and are not written.
int make_act_tmap3_box(CUtensorMap* map, const void* base, int batch, int L, int CP,
                       int elem_bytes, int box_bytes, int box_rows) {
  EncodeTiledFn fn = encode_tiled();
  if (!fn) return CHM_ERR_CUDA;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return CHM_ERR_WORKSPACE;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(CP), static_cast<cuuint64_t>(L),
                              static_cast<cuuint64_t>(batch)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(CP) * elem_bytes,
                                 static_cast<cuuint64_t>(CP) * elem_bytes * L};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(box_bytes / elem_bytes),
                             static_cast<cuuint32_t>(box_rows), 1u};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  const CUresult r = fn(map, elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                             : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                        3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        box_bytes == 32   ? CU_TENSOR_MAP_SWIZZLE_32B
                        : box_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                          : CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? CHM_OK : CHM_ERR_CUDA;
}

// ---- MLP kernel dispatch over (act_t, CP, HP)
template <typename act_t, int CP, int HP>
int launch_mlp_t(const MlpArgs& a, int grid, cudaStream_t st, bool fast) {
  const int smem = MlpSmem<CP, HP>::kAlloc;
  LaunchTimer timer(kKMlp, st);
  if (fast) {
    auto k = mlp_kernel<act_t, CP, HP, true>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    k<<<grid, 128, smem, st>>>(a);
  } else {
    auto k = mlp_kernel<act_t, CP, HP, false>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    k<<<grid, 128, smem, st>>>(a);
  }
  return launch_status();
}

template <typename act_t>
int launch_mlp(const Dims& m, const MlpArgs& a, int grid, cudaStream_t st) {
  const bool fast = (m.mode == CHM_MODE_BF16);
  if (m.CP == ws::kC && m.HP == ws::kH) {
    // per-example tiles (the last tile of an example is partial)
    const int batch = static_cast<int>(a.rows / m.L);
    MlpArgs ae = a;
    ae.tpe = (m.L + kTileRows - 1) / kTileRows;
    ae.n_tiles = batch * ae.tpe;
    const int egrid = std::max(1, std::min(ae.n_tiles, device_sms()));
    MlpMaps tmap;
    // bf16 residual: the input tile is read and the output tile written by TMA
    CHM_TRY(make_act_tmap3_box(&tmap.res, a.X_in, batch, m.L, m.CP, sizeof(act_t), 128,
                               kTileRows));
    CHM_TRY(make_act_tmap3_box(&tmap.out, a.X_out, batch, m.L, m.CP, sizeof(act_t), 128,
                               kTileRows));
    LaunchTimer timer(kKMlp, st);
    auto go = [&](auto k, int smem) {
      cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      launch_k(true, k, dim3(egrid), dim3(ws::kThreads), smem, st, ae, tmap);
    };
    bool wide = false;
    if constexpr (sizeof(act_t) == 2) {
      if (fast && a.dil <= ws::kWideMaxDil) {
        // small dilation: one (128 + 2d)-row block per 64-channel step
        using Lay = ws::Layout<act_t, true>;
        CHM_TRY(make_act_tmap3_box(&tmap.stage, a.X_in, batch, m.L, m.CP, sizeof(act_t),
                                   Lay::kBoxBytes, ws::wide_rows(a.dil)));
        go(mlp_ws_kernel<act_t, true, true>, Lay::kAlloc);
        wide = true;
      }
    }
    if (!wide) {
      using Lay = ws::Layout<act_t, false>;
      CHM_TRY(make_act_tmap3_box(&tmap.stage, a.X_in, batch, m.L, m.CP, sizeof(act_t),
                                 Lay::kBoxBytes, kTileRows));
      if (fast) go(mlp_ws_kernel<act_t, true, false>, Lay::kAlloc);
      else go(mlp_ws_kernel<act_t, false, false>, Lay::kAlloc);
    }
    return launch_status();
  }
  if constexpr (sizeof(act_t) == 2) {
    if (fast && m.CP == wd::kCP && m.HP % 64 == 0 && m.HP <= 512) {
      // n_filters 256 in bf16: warp-specialised, weights streamed in stages
      LaunchTimer timer(kKMlp, st);
      const int wgrid = std::max(1, std::min(a.n_tiles, device_sms()));
      cudaFuncSetAttribute(mlp_wide_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(wd::kAlloc));
      launch_k(true, mlp_wide_kernel, dim3(wgrid), dim3(wd::kThreads), wd::kAlloc, st, a);
      return launch_status();
    }
  }
  if (m.CP == 256 || m.HP > 256) {
    // wide models: weights streamed chunk by chunk
    LaunchTimer timer(kKMlp, st);
    auto go = [&](auto k, int smem) {
      cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      k<<<grid, 256, smem, st>>>(a);
    };
    auto pick = [&](auto cp) {
      constexpr int CPc = decltype(cp)::value;
      const int smem = static_cast<int>(StreamSmem<CPc>::kAlloc);
      if (fast) go(mlp_stream_kernel<act_t, CPc, true>, smem);
      else go(mlp_stream_kernel<act_t, CPc, false>, smem);
    };
    if (m.CP == 64) pick(std::integral_constant<int, 64>{});
    else if (m.CP == 128) pick(std::integral_constant<int, 128>{});
    else if (m.CP == 256) pick(std::integral_constant<int, 256>{});
    else return CHM_ERR_UNSUPPORTED;
    return launch_status();
  }
  if (m.CP == 64) {
    switch (m.HP) {
      case 64: return launch_mlp_t<act_t, 64, 64>(a, grid, st, fast);
      case 128: return launch_mlp_t<act_t, 64, 128>(a, grid, st, fast);
      case 192: return launch_mlp_t<act_t, 64, 192>(a, grid, st, fast);
      case 256: return launch_mlp_t<act_t, 64, 256>(a, grid, st, fast);
    }
  } else if (m.CP == 128) {
    switch (m.HP) {
      case 128: return launch_mlp_t<act_t, 128, 128>(a, grid, st, fast);
      case 192: return launch_mlp_t<act_t, 128, 192>(a, grid, st, fast);
      case 256: return launch_mlp_t<act_t, 128, 256>(a, grid, st, fast);
    }
  }
  return CHM_ERR_UNSUPPORTED;
}

// Per-example statistics with each thread reading the three conv rows of its
// positions directly (any activation type).
template <typename act_t>
int launch_stats_direct(const Dims& m, const act_t* X, const float* convw, int dil, int batch,
                        float2* stats, bool pdl, cudaStream_t st) {
  LaunchTimer timer(kKStats, st);
  if (m.CP == 64) {
    launch_k(pdl, stats_example_kernel<act_t, 64>, dim3(batch), dim3(kStats2Threads), 0, st, X,
             convw, dil, m.L, m.C, 1e-3f, stats);
  } else if (m.CP == 128) {
    launch_k(pdl, stats_example_kernel<act_t, 128>, dim3(batch), dim3(kStats2Threads), 0, st, X,
             convw, dil, m.L, m.C, 1e-3f, stats);
  } else if (m.CP == 256) {
    launch_k(pdl, stats_example_kernel<act_t, 256>, dim3(batch), dim3(kStats2Threads), 0, st, X,
             convw, dil, m.L, m.C, 1e-3f, stats);
  } else {
    return CHM_ERR_UNSUPPORTED;
  }
  return launch_status();
}

template <typename act_t>
int launch_stats(const Dims& m, const act_t* X, const float* convw, int dil, int batch,
                 float2* stats, bool pdl, cudaStream_t st) {
  if constexpr (sizeof(act_t) == 2) {
    // segment length: long segments amortise the two halo rows, short ones
    // avoid dead slots when the chains are short (large dilation); pick the
    // length with the fewest load slots plus per-segment overhead
    const int K = (m.L + dil - 1) / dil;            // longest chain
    // chains of at most 4 rows (d >= L / 4): the halo rows outnumber the
    // chain rows, so read the three rows of each position directly
    if (K <= 4) return launch_stats_direct<act_t>(m, X, convw, dil, batch, stats, pdl, st);
    static const int kLens[] = {4, 6, 8, 9, 12};
    int kS = 4;
    long best = -1;
    for (int len : kLens) {
      const long nkb = (K + len - 1) / len;
      const long cost = nkb * (len + 2) + 3 * nkb;
      if (best < 0 || cost < best) {
        best = cost;
        kS = len;
      }
    }
    const int n_kb = (K + kS - 1) / kS;
    LaunchTimer timer(kKStats, st);
    auto go = [&](auto kern, uint32_t smem) {
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem));
      launch_k(pdl, kern, dim3(batch), dim3(kStatsChainThreads), smem, st,
               reinterpret_cast<const __nv_bfloat16*>(X), convw, dil, m.L, m.C, n_kb, 1e-3f,
               stats);
    };
    auto pick = [&](auto cp) {
      constexpr int CPc = decltype(cp)::value;
      switch (kS) {
        case 4: go(stats_async_kernel<CPc, 4>, stats_async_smem_bytes<4>()); break;
        case 6: go(stats_async_kernel<CPc, 6>, stats_async_smem_bytes<6>()); break;
        case 8: go(stats_async_kernel<CPc, 8>, stats_async_smem_bytes<8>()); break;
        case 9: go(stats_async_kernel<CPc, 9>, stats_async_smem_bytes<9>()); break;
        default: go(stats_async_kernel<CPc, 12>, stats_async_smem_bytes<12>()); break;
      }
    };
    if (m.CP == 64) {
      pick(std::integral_constant<int, 64>{});
    } else if (m.CP == 128) {
      pick(std::integral_constant<int, 128>{});
    } else if (m.CP == 256) {
      pick(std::integral_constant<int, 256>{});
    } else {
      return CHM_ERR_UNSUPPORTED;
    }
    return launch_status();
  }
  return launch_stats_direct<act_t>(m, X, convw, dil, batch, stats, pdl, st);
}

// The whole forward for `batch` rows whose stem input is `in` (kind kIn).
template <typename act_t>
int run_forward_t(const Dims& m, const PackLayout& pl, const uint8_t* packed, int batch, int kIn,
                  const StemInput& in, const float* x_ctl, float* profile, float* logcounts,
                  uint8_t* ws, cudaStream_t st) {
  const FwdLayout f = fwd_layout(m, batch);
  float2* stats = reinterpret_cast<float2*>(ws + f.stats);
  int* status = reinterpret_cast<int*>(ws + f.status);
  act_t* xa = reinterpret_cast<act_t*>(ws + f.xa);
  act_t* xb = reinterpret_cast<act_t*>(ws + f.xb);

  // stem (tcgen05 im2col GEMM)
  const long long rows = (long long)batch * m.L;
  const int n_tiles = static_cast<int>((rows + kTileRows - 1) / kTileRows);
  {
    const float* bias = reinterpret_cast<const float*>(packed + pl.stem_b);
    const uint8_t* wpk = packed + pl.stem_pk;
    const bool split = (kIn == kInDense) && m.mode == CHM_MODE_FP32;
    LaunchTimer timer(kKStem, st);
    if (sizeof(act_t) == 2 && (m.CP == 128 || m.CP == 256) && !split) {
      // per-example tiles, TMA-stored output; one launch per 128 output channels
      CUtensorMap tmap;
      CHM_TRY(make_act_tmap3(&tmap, xa, batch, m.L, m.CP));
      const int tiles = batch * ((m.L + kTileRows - 1) / kTileRows);
      const int tgrid =
          std::max(1, std::min((tiles + sm2::kGroups - 1) / sm2::kGroups, device_sms()));
      const int tsmem = static_cast<int>(sm2::smem_bytes(1));
      for (int c_off = 0; c_off < m.CP; c_off += 128) {
        auto go = [&](auto k) {
          cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, tsmem);
          k<<<tgrid, sm2::kThreads, tsmem, st>>>(in, wpk, bias, tmap, batch, m.L, m.C, m.CP,
                                                 c_off, tiles, status);
        };
        if (kIn == kInDense) go(stem_tc_kernel<kInDense, 1>);
        else if (kIn == kInBases) go(stem_tc_kernel<kInBases, 1>);
        else go(stem_tc_kernel<kInIsm, 1>);
        CHM_TRY(launch_status());
      }
    } else if (sizeof(act_t) == 4 && (m.CP == 128 || m.CP == 256)) {
      // fp32 mode: the same tcgen05 stem with an fp32 output tile (two
      // warpgroups per CTA); dense fp32 input as bf16 hi + lo (three MMA terms)
      CUtensorMap tmap;
      CHM_TRY(make_act_tmap3_box(&tmap, xa, batch, m.L, m.CP, 4, 128, kTileRows));
      const int tiles = batch * ((m.L + kTileRows - 1) / kTileRows);
      constexpr int kG = sm2::groups_for(4);
      const int tgrid = std::max(1, std::min((tiles + kG - 1) / kG, device_sms()));
      const int splits = split ? 2 : 1;
      const int tsmem = static_cast<int>(sm2::smem_bytes(splits, 4));
      for (int c_off = 0; c_off < m.CP; c_off += 128) {
        auto go = [&](auto k) {
          cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, tsmem);
          k<<<tgrid, 128 * kG, tsmem, st>>>(in, wpk, bias, tmap, batch, m.L, m.C, m.CP, c_off,
                                            tiles, status);
        };
        if (kIn == kInDense) {
          if (split) go(stem_tc_kernel<kInDense, 2, float>);
          else go(stem_tc_kernel<kInDense, 1, float>);
        } else if (kIn == kInBases) {
          go(stem_tc_kernel<kInBases, 1, float>);
        } else {
          go(stem_tc_kernel<kInIsm, 1, float>);
        }
        CHM_TRY(launch_status());
      }
    } else {
    const int smem = stem_smem_bytes(m.CP, split ? 2 : 1);
    const int sgrid = std::min(n_tiles, 2 * device_sms());
#define CHM_STEM(KIN, SPLITS)                                                             \
  do {                                                                                    \
    auto k = stem_mma_kernel<act_t, KIN, SPLITS>;                                         \
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);           \
    k<<<sgrid, sm::kThreads, smem, st>>>(in, wpk, bias, xa, rows, m.L, m.C, m.CP, n_tiles, \
                                         status);                                         \
  } while (0)
    if (kIn == kInDense) {
      if (split) CHM_STEM(kInDense, 2); else CHM_STEM(kInDense, 1);
    } else if (kIn == kInBases) {
      CHM_STEM(kInBases, 1);
    } else {
      CHM_STEM(kInIsm, 1);
    }
#undef CHM_STEM
    CHM_TRY(launch_status());
    }
  }
  // block stack
  const int grid = std::min(n_tiles, device_sms());
  for (int i = 0; i < m.n_layers; ++i) {
    const uint8_t* lw = packed + pl.layers + pl.layer_stride * i;
    const float* convw = reinterpret_cast<const float*>(lw + pl.l_convw);
    const int dil = 1 << i;
    CHM_TRY(launch_stats<act_t>(m, xa, convw, dil, batch, stats, /*pdl=*/true, st));
    MlpArgs a;
    a.X_in = xa;
    a.X_out = xb;
    a.stats = stats;
    a.w1 = lw + pl.l_w1;
    a.w2 = lw + pl.l_w2;
    a.convw = convw;
    a.dil = dil;
    a.L = m.L;
    a.C = m.C;
    a.rows = rows;
    a.n_tiles = n_tiles;
    a.tpe = 0;
    a.HP = m.HP;
    a.status = status;
    CHM_TRY(launch_mlp<act_t>(m, a, grid, st));
    std::swap(xa, xb);
  }
  // heads
  const int cph = head_cph(m);
  const bool split_a = (m.mode == CHM_MODE_FP32);
  HeadArgs h;
  h.status = status;
  h.X = xa;
  h.X_ctl = x_ctl;
  h.fb = packed + pl.head_pk;
  h.fbias = reinterpret_cast<const float*>(packed + pl.head_fb);
  h.lw = reinterpret_cast<const float*>(packed + pl.head_lw);
  h.lbias = reinterpret_cast<const float*>(packed + pl.head_lb);
  h.profile = profile;
  h.logcounts = logcounts;
  h.L = m.L; h.C = m.C; h.CP = m.CP; h.CPH = cph; h.n_ctl = m.n_ctl; h.n_out = m.n_out;
  h.n_groups = m.n_groups; h.T = m.T; h.Lout = m.Lout;
  h.batch = batch;
  if (sizeof(act_t) == 2 && m.n_ctl == 0 && (m.CP == 128 || m.CP == 256) && cph == m.CP &&
      m.n_groups <= hd3::kMaxGroups) {
    CUtensorMap tmap;
    CHM_TRY(make_act_tmap3(&tmap, xa, batch, m.L, m.CP));
    const int hgrid = std::max(1, std::min(batch * m.n_out, device_sms()));
    LaunchTimer timer(kKProfile, st);
    auto go = [&](auto k) {
      cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, hd3::kAlloc);
      launch_k(true, k, dim3(hgrid), dim3(hd3::kThreads), hd3::kAlloc, st, h, tmap);
    };
    if (m.CP == 128) go(head_fused_kernel<128>);
    else go(head_fused_kernel<256>);
    CHM_TRY(launch_status());
  } else if (!(cph == 256 && split_a)) {
    const int smem = head_smem_bytes(cph, split_a ? 2 : 1);
    dim3 hgrid(m.n_out, batch);
    LaunchTimer timer(kKProfile, st);
    if (split_a) {
      auto k = head_kernel<act_t, 2>;
      cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      k<<<hgrid, hd::kThreads, smem, st>>>(h);
    } else {
      auto k = head_kernel<act_t, 1>;
      cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      k<<<hgrid, hd::kThreads, smem, st>>>(h);
    }
    CHM_TRY(launch_status());
  } else {
    const int cin = m.C + m.n_ctl;
    const int smem = (cin * kHeadWin + kHeadWarps * kHeadJ) * 4;
    auto k = profile_head_kernel<act_t>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    dim3 grid_h((m.Lout + kHeadJ - 1) / kHeadJ, batch);
    {
      LaunchTimer timer(kKProfile, st);
      k<<<grid_h, kHeadWarps * 32, smem, st>>>(
          xa, x_ctl, reinterpret_cast<const float*>(packed + pl.head_f),
          reinterpret_cast<const float*>(packed + pl.head_fb), profile, m.L, m.C, m.CP, m.n_ctl,
          m.n_out, m.T, m.Lout);
    }
    CHM_TRY(launch_status());
    {
      LaunchTimer timer(kKCount, st);
      count_head_kernel<act_t><<<batch, 256, 0, st>>>(
          xa, x_ctl, reinterpret_cast<const float*>(packed + pl.head_lw),
          reinterpret_cast<const float*>(packed + pl.head_lb), logcounts, m.L, m.C, m.CP,
          m.n_ctl, m.n_groups, m.T);
    }
    CHM_TRY(launch_status());
  }
  return CHM_OK;
}

int run_forward(const Dims& m, const uint8_t* packed, int batch, int kIn, const StemInput& in,
                const float* x_ctl, float* profile, float* logcounts, uint8_t* ws,
                cudaStream_t st) {
  const PackLayout pl = pack_layout(m);
  if (m.mode == CHM_MODE_BF16)
    return run_forward_t<__nv_bfloat16>(m, pl, packed, batch, kIn, in, x_ctl, profile, logcounts,
                                        ws, st);
  return run_forward_t<float>(m, pl, packed, batch, kIn, in, x_ctl, profile, logcounts, ws, st);
}

int validate(const chm_model_desc* d) {
  if (!d) return CHM_ERR_INVALID_ARGUMENT;
  if (d->n_filters < 1 || d->n_layers < 0 || d->n_layers > 24 || d->expansion < 1 ||
      d->n_outputs < 1 || d->n_groups < 1 || d->n_control_tracks < 0 || d->trimming < 0 ||
      d->seq_len < 1)
    return CHM_ERR_INVALID_ARGUMENT;
  if (d->mode != CHM_MODE_FP32 && d->mode != CHM_MODE_BF16) return CHM_ERR_INVALID_ARGUMENT;
  if (d->seq_len - 2 * d->trimming < 1) return CHM_ERR_UNSUPPORTED;
  const Dims m = dims_of(d);
  if (m.CP > 256 || m.HP > 512) return CHM_ERR_UNSUPPORTED;
  const int cin = m.C + m.n_ctl;
  if (cin > 256) return CHM_ERR_UNSUPPORTED;
  if ((cin * kHeadWin + kHeadWarps * kHeadJ) * 4 > 227 * 1024 && head_cph(m) == 256 &&
      m.mode == CHM_MODE_FP32)
    return CHM_ERR_UNSUPPORTED;
  return CHM_OK;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

size_t ism_len(const Dims& m) { return (size_t)m.n_out * m.Lout; }

struct IsmLayout {
  size_t fwd, ref_prof, ref_prob, ref_lc, ref_pw, mut_prof, mut_lc, total;
};

IsmLayout ism_layout(const Dims& m, int n_seqs, int mb) {
  IsmLayout l;
  size_t o = 0;
  l.fwd = o; o = align_up(o + fwd_layout(m, std::max(n_seqs, mb)).total);
  l.ref_prof = o; o = align_up(o + (size_t)n_seqs * ism_len(m) * 4);
  l.ref_prob = o; o = align_up(o + (size_t)n_seqs * ism_len(m) * 4);
  l.ref_lc = o; o = align_up(o + (size_t)n_seqs * m.n_groups * 4);
  l.ref_pw = o; o = align_up(o + (size_t)n_seqs * 4);
  l.mut_prof = o; o = align_up(o + (size_t)mb * ism_len(m) * 4);
  l.mut_lc = o; o = align_up(o + (size_t)mb * m.n_groups * 4);
  l.total = o;
  return l;
}

constexpr int kVariantChunk = 1024;

struct VarLayout {
  size_t fwd, ref_prof, ref_prob, ref_lc, alt_prof, alt_lc, total;
  int chunk;
};

VarLayout var_layout(const Dims& m, int n_pairs) {
  VarLayout l;
  l.chunk = std::max(1, std::min(n_pairs, kVariantChunk));
  size_t o = 0;
  l.fwd = o; o = align_up(o + fwd_layout(m, l.chunk).total);
  l.ref_prof = o; o = align_up(o + (size_t)l.chunk * ism_len(m) * 4);
  l.ref_prob = o; o = align_up(o + (size_t)l.chunk * ism_len(m) * 4);
  l.ref_lc = o; o = align_up(o + (size_t)l.chunk * m.n_groups * 4);
  l.alt_prof = o; o = align_up(o + (size_t)l.chunk * ism_len(m) * 4);
  l.alt_lc = o; o = align_up(o + (size_t)l.chunk * m.n_groups * 4);
  l.total = o;
  return l;
}

Dims block_dims(int C, int H, int x_dtype) {
  Dims m{};
  m.C = C;
  m.CP = pad_channels(C);
  m.H = H;
  m.HP = round64(H);
  m.mode = (x_dtype == CHM_INPUT_BF16) ? CHM_MODE_BF16 : CHM_MODE_FP32;
  m.rs = 1.f;
  return m;
}

bool block_supported(int C, int H) {
  return C >= 1 && H >= C && pad_channels(C) <= 256 && round64(H) <= 512;
}

struct BlockWsLayout {
  size_t status, stats, xin, xout, total;
};

BlockWsLayout block_ws_layout(const Dims& m, int batch) {
  BlockWsLayout b;
  size_t o = 0;
  b.status = o; o = align_up(o + 256);
  b.stats = o; o = align_up(o + (size_t)batch * 8);
  const size_t act = (m.C == m.CP) ? 0 : (size_t)batch * m.L * m.CP * m.act_bytes();
  b.xin = o; o = align_up(o + act);
  b.xout = o; o = align_up(o + act);
  b.total = o;
  return b;
}

template <typename act_t>
int run_block_t(const Dims& m, int batch, int dil, const uint8_t* packed, const act_t* x,
                act_t* out, uint8_t* ws, cudaStream_t st) {
  const BlockWsLayout bl = block_ws_layout(m, batch);
  const PackLayout pl = pack_layout(m);
  float2* stats = reinterpret_cast<float2*>(ws + bl.stats);
  const long long rows = (long long)batch * m.L;
  const act_t* xin = x;
  act_t* xout = out;
  if (m.C != m.CP) {
    act_t* pin = reinterpret_cast<act_t*>(ws + bl.xin);
    pad_channels_kernel<act_t><<<(unsigned)((rows * m.CP + 255) / 256), 256, 0, st>>>(
        x, pin, rows, m.C, m.CP);
    CHM_TRY(launch_status());
    xin = pin;
    xout = reinterpret_cast<act_t*>(ws + bl.xout);
  }
  const float* convw = reinterpret_cast<const float*>(packed + pl.l_convw);
  CHM_TRY(launch_stats<act_t>(m, xin, convw, dil, batch, stats, /*pdl=*/m.C != m.CP, st));
  const int n_tiles = static_cast<int>((rows + kTileRows - 1) / kTileRows);
  MlpArgs a;
  a.X_in = xin;
  a.X_out = xout;
  a.stats = stats;
  a.w1 = packed + pl.l_w1;
  a.w2 = packed + pl.l_w2;
  a.convw = convw;
  a.dil = dil;
  a.L = m.L;
  a.C = m.C;
  a.rows = rows;
  a.n_tiles = n_tiles;
  a.tpe = 0;
  a.HP = m.HP;
  a.status = reinterpret_cast<int*>(ws + bl.status);
  CHM_TRY(launch_mlp<act_t>(m, a, std::min(n_tiles, device_sms()), st));
  if (m.C != m.CP) {
    unpad_channels_kernel<act_t><<<(unsigned)((rows * m.C + 255) / 256), 256, 0, st>>>(
        xout, out, rows, m.C, m.CP);
    CHM_TRY(launch_status());
  }
  return CHM_OK;
}

// ---- static scratch of chm_forward_noalloc (see the header): device code
// could name the array directly; host code needs its device address, looked
// up once per device with that device current.
static __device__ __align__(256) uint8_t g_noalloc_scratch[CHM_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mutex;
void* g_noalloc_base[kMaxDevices] = {};

int noalloc_scratch(uint8_t** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CHM_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return CHM_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_base[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return CHM_ERR_CUDA;
    g_noalloc_base[dev] = p;
  }
  // the forward wants a 1024-byte-aligned workspace
  *out = reinterpret_cast<uint8_t*>(align_up(reinterpret_cast<uintptr_t>(g_noalloc_base[dev])));
  return CHM_OK;
}

}  // namespace

// ====================================================================== ABI
extern "C" {

int32_t chm_abi_version(void) { return CHM_ABI_VERSION; }

const char* chm_error_string(int32_t s) {
  switch (s) {
    case CHM_OK: return "ok";
    case CHM_ERR_INVALID_ARGUMENT: return "invalid argument";
    case CHM_ERR_UNSUPPORTED: return "unsupported model configuration";
    case CHM_ERR_WORKSPACE: return "workspace or packed-weight buffer too small or misaligned";
    case CHM_ERR_LAUNCH: return "kernel launch failed";
    case CHM_ERR_DEVICE_TIMEOUT: return "a bounded device-side wait timed out";
    case CHM_ERR_CUDA: return "CUDA runtime error";
  }
  return "unknown status";
}

int32_t chm_validate(const chm_model_desc* desc) { return validate(desc); }

size_t chm_packed_weights_bytes(const chm_model_desc* desc) {
  if (validate(desc) != CHM_OK) return 0;
  return pack_layout(dims_of(desc)).total;
}

int32_t chm_pack_weights(const chm_model_desc* desc, const chm_params* p, void* packed,
                         size_t packed_bytes, chm_stream_t stream) {
  g_launches = 0;
  CHM_TRY(validate(desc));
  if (!p || !packed || !p->iconv_weight || !p->iconv_bias || !p->fconv_weight ||
      !p->fconv_bias || !p->linear_weight || !p->linear_bias)
    return CHM_ERR_INVALID_ARGUMENT;
  if (desc->n_layers > 0 && (!p->conv_weight || !p->linear1_weight || !p->linear2_weight))
    return CHM_ERR_INVALID_ARGUMENT;
  const Dims m = dims_of(desc);
  const PackLayout pl = pack_layout(m);
  if (packed_bytes < pl.total || !aligned(packed, kAlign)) return CHM_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* dst = static_cast<uint8_t*>(packed);
  auto copy = [&](const float* src, size_t off, long long n) -> int {
    copy_f32_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(
        src, reinterpret_cast<float*>(dst + off), n);
    return launch_status();
  };
  CHM_TRY(copy(p->iconv_weight, pl.stem_w, (long long)m.C * 4 * kStemTaps));
  pack_sw128_split_kernel<<<(m.CP * sm::kK + 255) / 256, 256, 0, st>>>(
      p->iconv_weight, m.C, 4 * kStemTaps, m.CP, sm::kK, kStemTaps, p->iconv_bias,
      dst + pl.stem_pk);
  CHM_TRY(launch_status());
  CHM_TRY(copy(p->iconv_bias, pl.stem_b, m.C));
  for (int i = 0; i < m.n_layers; ++i) {
    if (!p->conv_weight[i] || !p->linear1_weight[i] || !p->linear2_weight[i])
      return CHM_ERR_INVALID_ARGUMENT;
    uint8_t* lw = dst + pl.layers + pl.layer_stride * i;
    pack_convw_kernel<<<(3 * m.CP + 255) / 256, 256, 0, st>>>(
        p->conv_weight[i], m.C, m.CP, reinterpret_cast<float*>(lw + pl.l_convw));
    CHM_TRY(launch_status());
    pack_sw128_kernel<<<(m.HP * m.CP + 255) / 256, 256, 0, st>>>(
        p->linear1_weight[i], m.H, m.C, m.HP, m.CP, 1.0f, lw + pl.l_w1);
    CHM_TRY(launch_status());
    // residual_scale folded into linear2 before the bf16 cast
    // (upstream cheri.py:1021-1024)
    pack_sw128_kernel<<<(m.CP * m.HP + 255) / 256, 256, 0, st>>>(
        p->linear2_weight[i], m.C, m.H, m.CP, m.HP, m.rs, lw + pl.l_w2);
    CHM_TRY(launch_status());
  }
  const long long cin = (long long)m.C + m.n_ctl;
  CHM_TRY(copy(p->fconv_weight, pl.head_f, (long long)m.n_out * cin * kHeadTaps));
  CHM_TRY(copy(p->fconv_bias, pl.head_fb, m.n_out));
  {
    const long long n = (long long)m.n_out * hd::kNP * head_cph(m);
    const bool count_rows = (m.n_ctl == 0 && m.n_groups <= hd3::kMaxGroups);
    pack_head_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(
        p->fconv_weight, m.n_out, (int)cin, kHeadTaps, hd::kNP, head_cph(m),
        count_rows ? p->linear_weight : nullptr, m.n_groups, dst + pl.head_pk);
    CHM_TRY(launch_status());
  }
  CHM_TRY(copy(p->linear_weight, pl.head_lw,
               (long long)m.n_groups * (m.C + (m.n_ctl > 0 ? 1 : 0))));
  CHM_TRY(copy(p->linear_bias, pl.head_lb, m.n_groups));
  return CHM_OK;
}

size_t chm_forward_workspace_bytes(const chm_model_desc* desc, int32_t batch) {
  if (validate(desc) != CHM_OK || batch < 1) return 0;
  return fwd_layout(dims_of(desc), batch).total;
}

static int forward_common(const chm_model_desc* desc, const void* packed, int32_t batch, int kIn,
                          const StemInput& in, const float* x_ctl, float* profile,
                          float* logcounts, void* ws, size_t ws_bytes, chm_stream_t stream) {
  g_launches = 0;
  CHM_TRY(validate(desc));
  if (batch < 0 || !packed || !profile || !logcounts || !ws) return CHM_ERR_INVALID_ARGUMENT;
  if (batch == 0) return CHM_OK;
  if (desc->n_control_tracks > 0 && !x_ctl) return CHM_ERR_INVALID_ARGUMENT;
  const Dims m = dims_of(desc);
  if (ws_bytes < fwd_layout(m, batch).total || !aligned(ws, kAlign) || !aligned(packed, kAlign))
    return CHM_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(ws, 0, sizeof(int), st) != cudaSuccess) return CHM_ERR_CUDA;
  return run_forward(m, static_cast<const uint8_t*>(packed), batch, kIn, in, x_ctl, profile,
                     logcounts, static_cast<uint8_t*>(ws), st);
}

int32_t chm_forward(const chm_model_desc* desc, const void* packed, int32_t batch, const void* x,
                    int32_t input_dtype, const float* x_ctl, float* profile, float* logcounts,
                    void* workspace, size_t workspace_bytes, chm_stream_t stream) {
  if (!x && batch > 0) return CHM_ERR_INVALID_ARGUMENT;
  if (input_dtype != CHM_INPUT_F32 && input_dtype != CHM_INPUT_BF16)
    return CHM_ERR_INVALID_ARGUMENT;
  StemInput in{};
  in.x = x;
  in.x_bf16 = (input_dtype == CHM_INPUT_BF16);
  return forward_common(desc, packed, batch, kInDense, in, x_ctl, profile, logcounts, workspace,
                        workspace_bytes, stream);
}

int32_t chm_forward_noalloc(const chm_model_desc* desc, const void* packed, int32_t batch,
                            const void* x, int32_t input_dtype, const float* x_ctl,
                            float* profile, float* logcounts, chm_stream_t stream) {
  CHM_TRY(validate(desc));
  if (batch < 0) return CHM_ERR_INVALID_ARGUMENT;
  const size_t usable = CHM_NOALLOC_SCRATCH_BYTES - kAlign;   // after aligning the base
  const size_t need = batch > 0 ? fwd_layout(dims_of(desc), batch).total : 0;
  if (need > usable) {
    fprintf(stderr,
            "cherimoya_b200: chm_forward_noalloc: a batch of %d needs %zu bytes of scratch; "
            "the static scratch holds %zu (split the batch)\n",
            batch, need, usable);
    return CHM_ERR_WORKSPACE;
  }
  uint8_t* ws = nullptr;
  CHM_TRY(noalloc_scratch(&ws));
  return chm_forward(desc, packed, batch, x, input_dtype, x_ctl, profile, logcounts, ws, usable,
                     stream);
}

int32_t chm_forward_bases(const chm_model_desc* desc, const void* packed, int32_t batch,
                          const int8_t* bases, const float* x_ctl, float* profile,
                          float* logcounts, void* workspace, size_t workspace_bytes,
                          chm_stream_t stream) {
  if (!bases && batch > 0) return CHM_ERR_INVALID_ARGUMENT;
  StemInput in{};
  in.bases = bases;
  return forward_common(desc, packed, batch, kInBases, in, x_ctl, profile, logcounts, workspace,
                        workspace_bytes, stream);
}

size_t chm_ism_workspace_bytes(const chm_model_desc* desc, int32_t n_seqs, int32_t mutant_batch) {
  if (validate(desc) != CHM_OK || n_seqs < 1 || mutant_batch < 1) return 0;
  return ism_layout(dims_of(desc), n_seqs, mutant_batch).total;
}

int32_t chm_ism(const chm_model_desc* desc, const void* packed, int32_t n_seqs,
                const int8_t* bases, int32_t start, int32_t end, int32_t mutant_batch,
                float* d_logcount, float* jsd, void* workspace, size_t workspace_bytes,
                chm_stream_t stream) {
  return chm_ism_ex(desc, packed, n_seqs, bases, start, end, mutant_batch, d_logcount, jsd,
                    nullptr, workspace, workspace_bytes, stream);
}

int32_t chm_ism_ex(const chm_model_desc* desc, const void* packed, int32_t n_seqs,
                   const int8_t* bases, int32_t start, int32_t end, int32_t mutant_batch,
                   float* d_logcount, float* jsd, float* d_profile_wrapper, void* workspace,
                   size_t workspace_bytes, chm_stream_t stream) {
  CHM_TRY(validate(desc));
  if (n_seqs < 0 || !packed || !bases || !d_logcount || !jsd || !workspace || mutant_batch < 1)
    return CHM_ERR_INVALID_ARGUMENT;
  if (n_seqs == 0) return CHM_OK;
  if (desc->n_control_tracks > 0) return CHM_ERR_UNSUPPORTED;
  if (start < 0 || end > desc->seq_len || end <= start) return CHM_ERR_INVALID_ARGUMENT;
  const Dims m = dims_of(desc);
  const IsmLayout il = ism_layout(m, n_seqs, mutant_batch);
  if (workspace_bytes < il.total || !aligned(workspace, kAlign) || !aligned(packed, kAlign))
    return CHM_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const uint8_t* pk = static_cast<const uint8_t*>(packed);
  float* ref_prof = reinterpret_cast<float*>(ws + il.ref_prof);
  float* ref_prob = reinterpret_cast<float*>(ws + il.ref_prob);
  float* ref_lc = reinterpret_cast<float*>(ws + il.ref_lc);
  float* ref_pw = d_profile_wrapper ? reinterpret_cast<float*>(ws + il.ref_pw) : nullptr;
  float* mut_prof = reinterpret_cast<float*>(ws + il.mut_prof);
  float* mut_lc = reinterpret_cast<float*>(ws + il.mut_lc);
  uint8_t* fws = ws + il.fwd;
  long long launches = 0;
  if (cudaMemsetAsync(ws, 0, sizeof(int), st) != cudaSuccess) return CHM_ERR_CUDA;

  StemInput rin{};
  rin.bases = bases;
  g_launches = 0;
  CHM_TRY(run_forward(m, pk, n_seqs, kInBases, rin, nullptr, ref_prof, ref_lc, fws, st));
  launches += g_launches;
  const int len = static_cast<int>(ism_len(m));
  softmax_rows_kernel<<<n_seqs, 256, 0, st>>>(ref_prof, ref_prob, len, ref_pw);
  CHM_TRY(launch_status());
  const int W = end - start;
  const long long total = (long long)n_seqs * W * 3;
  for (long long m0 = 0; m0 < total; m0 += mutant_batch) {
    const int nb = static_cast<int>(std::min<long long>(mutant_batch, total - m0));
    StemInput min{};
    min.bases = bases;
    min.mut0 = m0;
    min.ism_start = start;
    min.ism_width = W;
    g_launches = 0;
    CHM_TRY(run_forward(m, pk, nb, kInIsm, min, nullptr, mut_prof, mut_lc, fws, st));
    launches += g_launches;
    ScoreArgs sa{};
    sa.logits = mut_prof;
    sa.ref_probs = ref_prob;
    sa.lc = mut_lc;
    sa.lc_ref = ref_lc;
    sa.len = len;
    sa.n_groups = m.n_groups;
    sa.mut0 = m0;
    sa.per_ref = 3 * W;
    sa.ism = 1;
    sa.ism_start = start;
    sa.ism_width = W;
    sa.bases = bases;
    sa.L = m.L;
    sa.d_logcount = d_logcount;
    sa.jsd = jsd;
    sa.pw_ref = ref_pw;
    sa.d_pw = d_profile_wrapper;
    {
      LaunchTimer timer(kKScore, st);
      score_kernel<<<nb, 256, 0, st>>>(sa);
    }
    CHM_TRY(launch_status());
    ++launches;
  }
  {
    const long long n = (long long)n_seqs * W;
    ism_fill_ref_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(bases, m.L, start, W,
                                                                     m.n_groups, n_seqs,
                                                                     d_logcount, jsd,
                                                                     d_profile_wrapper);
    CHM_TRY(launch_status());
    launches += 2;
  }
  g_launches = launches;
  return CHM_OK;
}

int32_t chm_wrapper_epilogue(const chm_model_desc* desc, int32_t batch, const float* profile,
                             const float* logcounts, const int32_t* group_sizes,
                             float* expected_counts, float* profile_wrapper,
                             void* workspace, size_t workspace_bytes, chm_stream_t stream) {
  CHM_TRY(validate(desc));
  if (batch < 0 || !profile || !logcounts) return CHM_ERR_INVALID_ARGUMENT;
  if (batch == 0) return CHM_OK;
  const Dims m = dims_of(desc);
  const size_t len = (size_t)m.n_out * m.Lout;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (expected_counts) {
    if (!group_sizes || m.n_groups > kMaxEpilogueGroups) return CHM_ERR_INVALID_ARGUMENT;
    GroupOffsets go{};
    for (int g = 0; g < m.n_groups; ++g) {
      if (group_sizes[g] < 1) return CHM_ERR_INVALID_ARGUMENT;
      go.off[g + 1] = go.off[g] + group_sizes[g];
    }
    if (go.off[m.n_groups] != m.n_out) return CHM_ERR_INVALID_ARGUMENT;
    expected_counts_kernel<<<dim3(m.n_groups, batch), 256, 0, st>>>(
        profile, logcounts, m.n_out, m.Lout, m.n_groups, go, expected_counts);
    CHM_TRY(launch_status());
  }
  if (profile_wrapper) {
    // the softmax itself goes to the caller's workspace (batch * len floats)
    if (!workspace || workspace_bytes < (size_t)batch * len * sizeof(float))
      return CHM_ERR_WORKSPACE;
    softmax_rows_kernel<<<batch, 256, 0, st>>>(profile, static_cast<float*>(workspace),
                                               static_cast<int>(len), profile_wrapper);
    CHM_TRY(launch_status());
  }
  return CHM_OK;
}

size_t chm_variant_workspace_bytes(const chm_model_desc* desc, int32_t n_pairs) {
  if (validate(desc) != CHM_OK || n_pairs < 1) return 0;
  return var_layout(dims_of(desc), n_pairs).total;
}

int32_t chm_variant(const chm_model_desc* desc, const void* packed, int32_t n_pairs,
                    const int8_t* ref_bases, const int8_t* alt_bases, float* d_logcount,
                    float* jsd, void* workspace, size_t workspace_bytes, chm_stream_t stream) {
  CHM_TRY(validate(desc));
  if (n_pairs < 0 || !packed || !ref_bases || !alt_bases || !d_logcount || !jsd || !workspace)
    return CHM_ERR_INVALID_ARGUMENT;
  if (n_pairs == 0) return CHM_OK;
  if (desc->n_control_tracks > 0) return CHM_ERR_UNSUPPORTED;
  const Dims m = dims_of(desc);
  const VarLayout vl = var_layout(m, n_pairs);
  if (workspace_bytes < vl.total || !aligned(workspace, kAlign) || !aligned(packed, kAlign))
    return CHM_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const uint8_t* pk = static_cast<const uint8_t*>(packed);
  float* ref_prof = reinterpret_cast<float*>(ws + vl.ref_prof);
  float* ref_prob = reinterpret_cast<float*>(ws + vl.ref_prob);
  float* ref_lc = reinterpret_cast<float*>(ws + vl.ref_lc);
  float* alt_prof = reinterpret_cast<float*>(ws + vl.alt_prof);
  float* alt_lc = reinterpret_cast<float*>(ws + vl.alt_lc);
  uint8_t* fws = ws + vl.fwd;
  const int len = static_cast<int>(ism_len(m));
  long long launches = 0;
  if (cudaMemsetAsync(ws, 0, sizeof(int), st) != cudaSuccess) return CHM_ERR_CUDA;
  for (int p0 = 0; p0 < n_pairs; p0 += vl.chunk) {
    const int nb = std::min(vl.chunk, n_pairs - p0);
    StemInput rin{};
    rin.bases = ref_bases + (long long)p0 * m.L;
    g_launches = 0;
    CHM_TRY(run_forward(m, pk, nb, kInBases, rin, nullptr, ref_prof, ref_lc, fws, st));
    launches += g_launches;
    StemInput ain{};
    ain.bases = alt_bases + (long long)p0 * m.L;
    g_launches = 0;
    CHM_TRY(run_forward(m, pk, nb, kInBases, ain, nullptr, alt_prof, alt_lc, fws, st));
    launches += g_launches;
    softmax_rows_kernel<<<nb, 256, 0, st>>>(ref_prof, ref_prob, len, nullptr);
    CHM_TRY(launch_status());
    ScoreArgs sa{};
    sa.logits = alt_prof;
    sa.ref_probs = ref_prob;
    sa.lc = alt_lc;
    sa.lc_ref = ref_lc;
    sa.len = len;
    sa.n_groups = m.n_groups;
    sa.mut0 = 0;
    sa.per_ref = 1;
    sa.ism = 0;
    sa.d_logcount = d_logcount + (long long)p0 * m.n_groups;
    sa.jsd = jsd + p0;
    score_kernel<<<nb, 256, 0, st>>>(sa);
    CHM_TRY(launch_status());
    launches += 2;
  }
  g_launches = launches;
  return CHM_OK;
}

size_t chm_block_packed_bytes(int32_t n_filters, int32_t hidden) {
  if (!block_supported(n_filters, hidden)) return 0;
  const Dims m = block_dims(n_filters, hidden, CHM_INPUT_F32);
  return pack_layout(m).layer_stride;
}

int32_t chm_pack_block(int32_t n_filters, int32_t hidden, float residual_scale,
                       const float* conv_weight, const float* linear1_weight,
                       const float* linear2_weight, void* packed, size_t packed_bytes,
                       chm_stream_t stream) {
  g_launches = 0;
  if (!block_supported(n_filters, hidden)) return CHM_ERR_UNSUPPORTED;
  if (!conv_weight || !linear1_weight || !linear2_weight || !packed)
    return CHM_ERR_INVALID_ARGUMENT;
  const Dims m = block_dims(n_filters, hidden, CHM_INPUT_F32);
  const PackLayout pl = pack_layout(m);
  if (packed_bytes < pl.layer_stride || !aligned(packed, kAlign)) return CHM_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* lw = static_cast<uint8_t*>(packed);
  pack_convw_kernel<<<(3 * m.CP + 255) / 256, 256, 0, st>>>(
      conv_weight, m.C, m.CP, reinterpret_cast<float*>(lw + pl.l_convw));
  CHM_TRY(launch_status());
  pack_sw128_kernel<<<(m.HP * m.CP + 255) / 256, 256, 0, st>>>(linear1_weight, m.H, m.C, m.HP,
                                                               m.CP, 1.0f, lw + pl.l_w1);
  CHM_TRY(launch_status());
  pack_sw128_kernel<<<(m.CP * m.HP + 255) / 256, 256, 0, st>>>(
      linear2_weight, m.C, m.H, m.CP, m.HP, residual_scale, lw + pl.l_w2);
  return launch_status();
}

size_t chm_block_workspace_bytes(int32_t batch, int32_t seq_len, int32_t n_filters,
                                 int32_t x_dtype) {
  if (batch < 1 || seq_len < 1 || n_filters < 1 || round64(n_filters) > 128) return 0;
  Dims m = block_dims(n_filters, n_filters, x_dtype);
  m.L = seq_len;
  return block_ws_layout(m, batch).total;
}

int32_t chm_block_forward(int32_t batch, int32_t seq_len, int32_t n_filters, int32_t hidden,
                          int32_t dilation, int32_t x_dtype, const void* packed, const void* x,
                          void* out, void* workspace, size_t workspace_bytes,
                          chm_stream_t stream) {
  g_launches = 0;
  if (!block_supported(n_filters, hidden)) return CHM_ERR_UNSUPPORTED;
  if (batch < 0 || seq_len < 1 || dilation < 0 || !packed || !workspace ||
      (x_dtype != CHM_INPUT_F32 && x_dtype != CHM_INPUT_BF16))
    return CHM_ERR_INVALID_ARGUMENT;
  if (batch == 0) return CHM_OK;
  if (!x || !out || x == out) return CHM_ERR_INVALID_ARGUMENT;
  Dims m = block_dims(n_filters, hidden, x_dtype);
  m.L = seq_len;
  if (workspace_bytes < block_ws_layout(m, batch).total || !aligned(workspace, kAlign) ||
      !aligned(packed, kAlign) || !aligned(x, 16) || !aligned(out, 16))
    return CHM_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (cudaMemsetAsync(ws, 0, sizeof(int), st) != cudaSuccess) return CHM_ERR_CUDA;
  const uint8_t* pk = static_cast<const uint8_t*>(packed);
  if (x_dtype == CHM_INPUT_BF16)
    return run_block_t<__nv_bfloat16>(m, batch, dilation, pk,
                                      static_cast<const __nv_bfloat16*>(x),
                                      static_cast<__nv_bfloat16*>(out), ws, st);
  return run_block_t<float>(m, batch, dilation, pk, static_cast<const float*>(x),
                            static_cast<float*>(out), ws, st);
}

int32_t chm_read_status(void* workspace, chm_stream_t stream) {
  if (!workspace) return CHM_ERR_INVALID_ARGUMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaStreamSynchronize(st) != cudaSuccess) return CHM_ERR_CUDA;
  int s = 0;
  if (cudaMemcpy(&s, workspace, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
    return CHM_ERR_CUDA;
  if (s != 0 && cudaMemset(workspace, 0, sizeof(int)) != cudaSuccess) return CHM_ERR_CUDA;
  return s;
}

int32_t chm_selftest_wait_timeout(void* workspace, size_t workspace_bytes,
                                  chm_stream_t stream) {
  if (!workspace || workspace_bytes < sizeof(int) || !aligned(workspace, sizeof(int)))
    return CHM_ERR_INVALID_ARGUMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(workspace, 0, sizeof(int), st) != cudaSuccess) return CHM_ERR_CUDA;
  wait_timeout_selftest_kernel<<<1, 32, 0, st>>>(static_cast<int*>(workspace));
  return launch_status();
}

int32_t chm_noalloc_read_status(chm_stream_t stream) {
  uint8_t* ws = nullptr;
  CHM_TRY(noalloc_scratch(&ws));
  return chm_read_status(ws, stream);
}

int64_t chm_last_launch_count(void) { return g_launches; }

void chm_timing_enable(int32_t enable) { g_timing.enabled = (enable != 0); }

int32_t chm_timing_collect(double* ms_per_class, int64_t* launches_per_class) {
  for (int c = 0; c < kKClasses; ++c) {
    if (ms_per_class) ms_per_class[c] = 0.0;
    if (launches_per_class) launches_per_class[c] = 0;
  }
  int status = CHM_OK;
  for (TimedLaunch& t : g_timing.pending) {
    float ms = 0.f;
    if (cudaEventSynchronize(t.stop) != cudaSuccess ||
        cudaEventElapsedTime(&ms, t.start, t.stop) != cudaSuccess)
      status = CHM_ERR_CUDA;
    if (ms_per_class) ms_per_class[t.cls] += ms;
    if (launches_per_class) launches_per_class[t.cls] += 1;
    g_timing.pool.push_back(t.start);
    g_timing.pool.push_back(t.stop);
  }
  g_timing.pending.clear();
  return status;
}

}  // extern "C"
