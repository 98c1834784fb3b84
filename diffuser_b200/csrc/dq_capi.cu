// dq_capi.cu -- C ABI of the quantized-linear engine (include/dq_linear.h):
// argument validation, launch planning, TMA descriptors, and the standalone
// quantize / dequantize / split-K reduce kernels.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdint>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "../../include/dq_linear.h"
#include "../../include/dq_dit.h"
#include "dq_gemm.cuh"
#include "dq_gemm2.cuh"
#include "dq_bf16gemm2.cuh"
#include "dq_dit.cuh"
#include "dq_smallm.cuh"
#include "dq_smallm2.cuh"

#define DQ_VERSION_STRING "dqlinear-b200 0.1.0 (sm_100a)"

namespace dq {

// ------------------------------------------------------- standalone kernels
// NF4 -> bf16 and e4m3 -> bf16 over the whole flat weight (the staged chunk
// loops of dq_codec.cuh; 8 warps x 2 KB of staging per CTA), fp8 with a
// scalar tail for n % 16.
__global__ void __launch_bounds__(256)
    dequant_nf4_kernel(const uint4* __restrict__ packed, const void* __restrict__ absmax,
                       uint4* __restrict__ out, int64_t n_chunks, int scale_bf16) {
  __shared__ uint4 stage[8][128];
  dequant_nf4_chunks(packed, absmax, out, 0, n_chunks,
                     blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x,
                     static_cast<int64_t>(gridDim.x) * blockDim.x, stage[threadIdx.x >> 5], scale_bf16 != 0);
}

__global__ void __launch_bounds__(256)
    dequant_fp8_kernel(const uint8_t* __restrict__ w8, float scale, __nv_bfloat16* __restrict__ out,
                       int64_t n) {
  __shared__ uint4 stage[8][64];
  const float s = __bfloat162float(__float2bfloat16_rn(scale));
  const int64_t n16 = n / 16;
  const int64_t tid = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const int64_t nth = static_cast<int64_t>(gridDim.x) * blockDim.x;
  dequant_fp8_chunks(reinterpret_cast<const uint4*>(w8), s, reinterpret_cast<uint4*>(out), 0, n16,
                     tid, nth, stage[threadIdx.x >> 5]);
  for (int64_t i = n16 * 16 + tid; i < n; i += nth) {
    uint32_t o[2];
    fp8_decode_word(static_cast<uint32_t>(w8[i]), s, o);
    out[i] = __ushort_as_bfloat16(static_cast<unsigned short>(o[0] & 0xFFFFu));
  }
}

// Grid of an elementwise decode: four chunks per thread per pass, at most the
// CTAs that are resident at once (8 x 256 threads per SM).
static int decode_grid(int64_t chunks, int sms) {
  int64_t g = (chunks + 4 * 256 - 1) / (4 * 256);
  g = std::min<int64_t>(g, static_cast<int64_t>(sms) * 8);
  return static_cast<int>(std::max<int64_t>(g, 1));
}

template <typename T>
__device__ __forceinline__ float load_f32(const T* p, int64_t i);
template <>
__device__ __forceinline__ float load_f32<float>(const float* p, int64_t i) { return p[i]; }
template <>
__device__ __forceinline__ float load_f32<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
  return __bfloat162float(p[i]);
}

// NF4 quantizer: one warp per 64-element block, two elements per lane.
template <typename T>
__global__ void quantize_nf4_kernel(const T* __restrict__ w, uint8_t* __restrict__ packed,
                                    float* __restrict__ absmax, int64_t n_blocks) {
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t b = warp0; b < n_blocks; b += nwarps) {
    const float v0 = load_f32(w, b * 64 + 2 * lane);
    const float v1 = load_f32(w, b * 64 + 2 * lane + 1);
    float a = fmaxf(fabsf(v0), fabsf(v1));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    a = fmaxf(a, 1e-12f);
    const uint32_t c0 = nf4_code(__fdiv_rn(v0, a));
    const uint32_t c1 = nf4_code(__fdiv_rn(v1, a));
    packed[b * 32 + lane] = static_cast<uint8_t>((c0 << 4) | c1);
    if (lane == 0) absmax[b] = a;
  }
}

// fp8 quantizer, pass 1: max |w| as ordered float bits (non-negative floats
// order like their bit patterns).
template <typename T>
__global__ void absmax_kernel(const T* __restrict__ w, int64_t n, unsigned int* __restrict__ amax_bits) {
  float a = 0.f;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    a = fmaxf(a, fabsf(load_f32(w, i)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
  if ((threadIdx.x & 31) == 0) atomicMax(amax_bits, __float_as_uint(a));
}

__device__ __forceinline__ float fp8_scale_from_bits(unsigned int bits) {
  return __fdiv_rn(fmaxf(__uint_as_float(bits), 1e-12f), 448.0f);
}

// fp8 quantizer, pass 2: w8 = e4m3(w / scale).
template <typename T>
__global__ void quantize_fp8_kernel(const T* __restrict__ w, int64_t n, const unsigned int* amax_bits,
                                    uint8_t* __restrict__ w8) {
  const float scale = fp8_scale_from_bits(*amax_bits);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    w8[i] = f32_to_e4m3(__fdiv_rn(load_f32(w, i), scale));
}

// fp8 quantizer, pass 3: replace the max bits by the scale itself.
__global__ void finalize_fp8_scale_kernel(unsigned int* amax_bits_then_scale) {
  const float s = fp8_scale_from_bits(*amax_bits_then_scale);
  *reinterpret_cast<float*>(amax_bits_then_scale) = s;
}

// Column-parallel completion: thread r waits (bounded) until rank r has raised
// its flag in this rank's flag array to `epoch`; on expiry the device error
// word records DQ_ERR_TIMEOUT and the wait ends.
__global__ void tp_wait_kernel(const unsigned int* flags, int world, unsigned int epoch,
                               unsigned long long limit_ns) {
  const int r = threadIdx.x;
  if (r >= world) return;
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + r) : "memory");
    if (static_cast<int>(v - epoch) >= 0) return;
    if (globaltimer_ns() - t0 > limit_ns) {
      atomicOr(&g_dq_error, 1u << kErrTimeout);
      return;
    }
    __nanosleep(256);
  }
}

// Split-K: y[m, n] (row stride ldy) = bf16(sum_s partial[s][m, n] + bias);
// with a gated activation y[m, j] (j < N / 2) from the gate row
// 32 * (j / 16) + j % 16 and the up row 16 further (the gated row order).
__global__ void splitk_reduce_kernel(const float* __restrict__ part, int splits, int M, int N,
                                     const __nv_bfloat16* __restrict__ bias,
                                     __nv_bfloat16* __restrict__ y, int act, int64_t ldy) {
  const int64_t total = static_cast<int64_t>(M) * N;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  if (act_is_gated(act)) {
    const int no = N / 2;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
         i < static_cast<int64_t>(M) * no; i += stride) {
      const int64_t m = i / no;
      const int j = static_cast<int>(i - m * no);
      const int ng = 32 * (j / 16) + j % 16;
      float g = 0.f, u = 0.f;
      for (int s = 0; s < splits; ++s) {
        g += part[static_cast<size_t>(s) * total + m * N + ng];
        u += part[static_cast<size_t>(s) * total + m * N + ng + 16];
      }
      if (bias != nullptr) {
        g += __bfloat162float(bias[ng]);
        u += __bfloat162float(bias[ng + 16]);
      }
      y[m * ldy + j] = __float2bfloat16_rn(gated_value(g, u, act));
    }
    return;
  }
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total; i += stride) {
    float acc = 0.f;
    for (int s = 0; s < splits; ++s) acc += part[static_cast<size_t>(s) * total + i];
    const int64_t m = i / N, n = i - m * N;
    if (bias != nullptr) acc += __bfloat162float(bias[n]);
    y[m * ldy + n] = __float2bfloat16_rn(apply_act(acc, act));
  }
}

// ------------------------------------------------------------ device cache
// Per-device facts and one-time kernel set-up.  Host threads may call the
// library concurrently: every flag below is set (release) only after the
// values it guards are written under g_dev_mu, and is read (acquire) without
// the lock, so a reader that sees a flag also sees those values.
struct DeviceInfo {
  std::atomic<int> ok;  // 1 = probed
  int major = 0, minor = 0, sms = 0;
  // fused kernels, [variant: plain, column-parallel, gated][fmt][bm]
  std::atomic<int> smem_set[3][2][6];
  std::atomic<int> smem_set2[3][2][6];
  int max_pairs[3][2][6] = {};
  // bf16 pair GEMM, [column-parallel][decoded format + 1][bm]
  std::atomic<int> bf16_smem_set[2][3][6];
  int bf16_max_pairs[2][3][6] = {};
  std::atomic<int> smallm_set[3][2][3];    // small-M kernel, [fmt, or 2 = NF4 with bf16 scales][token tiles - 1][row groups 1/2/4]
  std::atomic<int> smallm2_set[2][2][3];   // small-M TMA-ring kernel, [fmt][CTAs per SM - 2][row groups]
  std::atomic<int> smallm2_mt2_set[2];     // ... with two token tiles, [fmt]
};

constexpr int kMaxDevices = 64;
static DeviceInfo g_dev[kMaxDevices];  // static storage: every flag starts at zero
static std::mutex g_dev_mu;
static std::atomic<int> g_override_bm{0}, g_override_splits{0}, g_override_pair{0};

// Runs init() once per flag (per device and kernel configuration), under the
// device mutex; the flag is raised only when init succeeds.
template <typename F>
static int once_per_device(std::atomic<int>& flag, F&& init) {
  if (flag.load(std::memory_order_acquire)) return DQ_OK;
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (flag.load(std::memory_order_relaxed)) return DQ_OK;
  const int rc = init();
  if (rc == DQ_OK) flag.store(1, std::memory_order_release);
  return rc;
}

static int current_device(DeviceInfo** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return DQ_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return DQ_ERR_CUDA;
  DeviceInfo& d = g_dev[dev];
  const int rc = once_per_device(d.ok, [&] {
    if (cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return static_cast<int>(DQ_ERR_CUDA);
    return static_cast<int>(DQ_OK);
  });
  if (rc != DQ_OK) return rc;
  *out = &d;
  if (d.major != 10) return DQ_ERR_ARCH;
  return DQ_OK;
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

static bool make_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint64_t inner,
                        uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                        CUtensorMapSwizzle swz) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// ----------------------------------------------------------- launch plan
struct Plan {
  bool pair = false;      // CTA-pair tiles (256 weight rows per tile)
  bool twophase = false;  // dequantize into bf16 scratch, then the bf16 pair GEMM
  bool smallm = false;    // decode-sized M: register-decode warp MMAs (smallm_kernel)
  bool ring = false;      // ... with the weight streamed through a TMA ring (smallm2_kernel)
  int r16 = 1;            // small-M: 16-row groups per CTA
  int cps = 2;            // small-M ring kernel: resident CTAs per SM
  int bm = 0, splits = 1, kb_per_split = 0;
  int m_tiles = 0, n_tiles = 0, tiles = 0, grid = 0;
  size_t ws = 0;
};

static int bm_index(int bm) {
  switch (bm) {
    case 16: return 0;
    case 32: return 1;
    case 64: return 2;
    case 128: return 3;
    case 192: return 4;
    case 256: return 5;
  }
  return -1;
}

// Relative per-SM throughput of each large-M tile shape (one-CTA BM=192 = 1),
// measured on B200 at x[4608,3072] . W[12288,3072]^T for both formats.
struct TileShape {
  bool pair;
  int bm;
  double eff;
};
static constexpr TileShape kShapes[] = {
    {false, 128, 0.72}, {false, 192, 1.0}, {false, 256, 0.97}, {true, 192, 0.93}, {true, 256, 1.13}};

// The small-M kernel serves M <= kSmallMMaxM (two 8-token tiles) with K a
// multiple of 128.
constexpr int64_t kSmallMMaxM = 16;
// Row groups (16 weight rows each) per small-M CTA, so one CTA's LUT fill and
// x loads serve more rows and more weight bytes are in flight per warp: the
// most that still give every SM a CTA (measured: four for NF4 with one token
// tile when that still leaves about two CTAs per SM -- 3072->18432 12.7 us
// against 16.9 with two, 4096->12288 15.9 against 14.2 -- two for fp8 and for
// two token tiles, whose registers run out).
static int smallm_r16(int fmt, int64_t M, int64_t N, int sms) {
  if (fmt == kFmtNF4 && M <= 8 && 2 * ((N + 63) / 64) >= 3 * static_cast<int64_t>(sms)) return 4;
  return (N + 31) / 32 >= sms ? 2 : 1;
}
// Row groups per CTA (R16) and resident CTAs per SM (CPS) of the TMA-ring
// small-M kernel: the configuration whose grid fills the largest share of the
// resident slots in one wave (measured, M = 1, NF4: 3072 -> 12288 at R16 = 2
// 15.3 us with two CTAs per SM, where the 384 CTAs need two waves, 10.6 us
// with three; 3072 -> 18432 11.6 us at R16 = 4 / CPS = 2, 15.0 us with three
// CTAs per SM, whose 288 CTAs then leave slots empty and have shallower rings).
// Beyond one wave at three CTAs per SM: R16 = 4, CPS = 3.
static void smallm2_config(int64_t N, int sms, bool gated, int* r16_out, int* cps_out) {
  double best = -1.0;
  *r16_out = 4;
  *cps_out = 3;
  for (int cps : {3, 2})
    for (int r16 : {4, 2, 1}) {
      if (gated && r16 == 1) continue;  // a gate / up pair of row groups per CTA
      const int64_t grid = (N + 16 * r16 - 1) / (16 * r16);
      const int64_t slots = static_cast<int64_t>(cps) * sms;
      if (grid > slots) continue;
      const double fill = static_cast<double>(grid) / static_cast<double>(slots);
      if (fill > best + 1e-9) {
        best = fill;
        *r16_out = r16;
        *cps_out = cps;
      }
    }
}
// The TMA-ring kernel takes NF4 block-scale tiles by TMA (rows of K / 64
// floats must be whole 16-byte units).  One 8-token tile: automatic up to four
// tokens (from about eight, every consumer lane reads x through an L1 that the
// ring's shared memory has mostly taken, and the register-stream kernel is
// faster: 3072 -> 18432 at M = 8, 16.7 against 13.9 us).  Two token tiles
// (9-16 tokens, x staged in the ring, 64-row CTAs two per SM): automatic when
// the grid fills at least 5/8 of those slots (measured, NF4 / fp8 at M = 16:
// 3072 -> 18432 18.4 / 16.9 us against 20.9 / 18.0, 4096 -> 12288 23.3 / 20.6
// against 25.6 / 20.6; 3072 -> 9216, one CTA per SM, 17.3 against 11.5).
constexpr int64_t kSmallM2AutoMaxM = 4;
static bool smallm2_shape_ok(int fmt, int64_t M, int64_t K) {
  return M <= 16 && (fmt == kFmtNF4 ? K % 256 == 0 : K % 128 == 0);
}

// Row groups per CTA of the register-stream small-M kernel; a gated
// activation needs its gate and up row groups in one CTA (an even count).
static int smallm_rows(int fmt, int64_t M, int64_t N, int sms, bool gated) {
  const int r16 = smallm_r16(fmt, M, N, sms);
  return gated ? std::max(r16, 2) : r16;
}

// Token count from which the two-phase plan is chosen: decoding the weight
// once (~N*K*2.6 bytes of HBM traffic) costs less than decoding it in every
// token tile, and the bf16 pair GEMM runs faster than the fused kernels.
constexpr int64_t kTwoPhaseMinM = 1024;

// Two-phase workspace: the bf16 weight [N, K], then one uint32 counter per
// weight group (at most one group per 256-row weight tile).
static size_t twophase_counter_offset(int64_t N, int64_t K) {
  return (static_cast<size_t>(N) * K * 2 + 255) & ~static_cast<size_t>(255);
}
static size_t twophase_counter_bytes(int n_tiles) {
  return (static_cast<size_t>(n_tiles + 1) * 4 + 255) & ~static_cast<size_t>(255);
}
// Weight tiles per group of the two-phase grouped order (16 x 256 rows: a
// group's bf16 weight stays in L2 while the token tiles sweep past it).
constexpr int kTwoPhaseGroupN = 16;

// max_split_ws: the most split-K scratch the caller can hold (the
// allocation-free entry point's built-in array): automatic plans split at most
// as far as their partial sums fit it; only a forced split count can exceed it.
static Plan make_plan(int fmt, int64_t M, int64_t N, int64_t K, int sms, bool allow_split = true,
                      bool allow_twophase = true, bool allow_smallm = true,
                      size_t max_split_ws = SIZE_MAX, bool gated = false) {
  Plan p;
  int long_k_split = 0;
  const int KB = static_cast<int>((K + 63) / 64);
  // 0 automatic, 1 one-CTA fused only, 2 CTA-pair fused only, 3 two-phase
  // only, 4 two-phase only with the dequantization as its own launch, 5 the
  // small-M kernel wherever it applies
  const int opair = g_override_pair.load();
  const int obm = g_override_bm.load();
  // Automatic for M <= 8 (one 8-token tile); for a second tile only with two
  // row groups per CTA -- with one, the fused kernel is faster there.  The
  // TMA-ring kernel wherever its shape rule holds (pair mode 6 forces the
  // register-stream kernel).
  if (allow_smallm && M <= kSmallMMaxM && K % 128 == 0 &&
      (opair == 5 || opair == 6 ||
       (opair == 0 && obm == 0 && g_override_splits.load() == 0 &&
        (M <= 8 || smallm_r16(fmt, M, N, sms) >= 2)))) {
    p.smallm = true;
    p.ring = smallm2_shape_ok(fmt, M, K) &&
             (opair == 5 || (opair == 0 && (M <= kSmallM2AutoMaxM ||
                                            (M > 8 && (N + 63) / 64 >= (5 * static_cast<int64_t>(sms)) / 4))));
    p.bm = M <= 8 ? 8 : 16;
    p.m_tiles = 1;
    int r16 = smallm_rows(fmt, M, N, sms, gated);
    if (p.ring) {
      if (M > 8) {  // two token tiles: x staged in the ring, 64-row CTAs, two per SM
        r16 = 4;
        p.cps = 2;
      } else {
        smallm2_config(N, sms, gated, &r16, &p.cps);
      }
    }
    p.r16 = r16;
    p.n_tiles = static_cast<int>((N + 16 * r16 - 1) / (16 * r16));
    p.tiles = p.n_tiles;
    p.grid = p.n_tiles;
    p.splits = 1;
    p.kb_per_split = KB;
    p.ws = 0;
    return p;
  }
  auto units_of = [&](bool pair) { return pair ? sms / 2 : sms; };
  auto n_tiles_of = [&](bool pair) { return static_cast<int>((N + (pair ? 255 : 127)) / (pair ? 256 : 128)); };
  const bool twophase = allow_twophase && M > 64 &&
                        (opair == 3 || opair == 4 || (opair == 0 && M >= kTwoPhaseMinM));
  if (twophase) {
    p.pair = true;
    p.twophase = true;
    if (obm >= 64 && bm_index(obm) >= 0) {
      p.bm = obm;
    } else {
      // fewest waves x tile time, each x-tile height weighted by its measured
      // throughput relative to BM = 256 (DiT shapes at M = 4096 / 4608: 192 runs
      // at 0.94 of it, 128 at 0.83), preferring the taller tile on ties
      p.bm = 256;
      double best = 1e30;
      constexpr struct { int bm; double eff; } kTwoPhaseShapes[] = {{256, 1.0}, {192, 0.94}, {128, 0.83}};
      for (const auto& c : kTwoPhaseShapes) {
        const int64_t tiles = ((M + c.bm - 1) / c.bm) * n_tiles_of(true);
        const double cost =
            static_cast<double>((tiles + units_of(true) - 1) / units_of(true)) * c.bm / c.eff;
        if (cost < best - 1e-9) { best = cost; p.bm = c.bm; }
      }
    }
  } else if (opair == 2 && M > 64) {
    p.pair = true;
    p.bm = (obm >= 64 && bm_index(obm) >= 0) ? obm : 256;
  } else if (obm > 0 && bm_index(obm) >= 0) {
    p.bm = obm;
  } else if (M <= 16) {
    p.bm = 16;
  } else if (M <= 32) {
    p.bm = 32;
  } else if (M <= 64) {
    p.bm = 64;
  } else if (M <= 128) {
    p.bm = 128;
  } else {
    // Minimize waves x tile time over the large-M shapes; CTA-pair shapes only
    // when they fill every SM pair without split-K.
    double best = 1e30;
    for (const TileShape& c : kShapes) {
      if (c.pair && opair == 1) continue;
      const int64_t tiles = ((M + c.bm - 1) / c.bm) * n_tiles_of(c.pair);
      const int units = units_of(c.pair);
      if (c.pair && tiles < units) continue;
      const double waves = static_cast<double>((tiles + units - 1) / units);
      const double cost = waves * (c.pair ? 256.0 : 128.0) * c.bm / ((c.pair ? 2.0 : 1.0) * c.eff);
      if (cost < best - 1e-9) {
        best = cost;
        p.pair = c.pair;
        p.bm = c.bm;
      }
    }
    // Long K on a partial wave: one-CTA tiles split in two K halves that fill
    // the SMs exactly once, costed at half a tile plus 15% for the f32 partials
    // and their reduce (measured at M = 512, 12288 -> 3072: 192-row tiles split
    // two ways 58.6 us against 75.2 for the unsplit 128-row grid; the
    // 3072-deep projections of that size stay unsplit, as measured fastest).
    if (allow_split && KB >= 128 && opair == 0 && obm == 0 && g_override_splits.load() == 0 &&
        static_cast<size_t>(2) * M * N * sizeof(float) <= max_split_ws) {
      for (const TileShape& c : kShapes) {
        if (c.pair) continue;
        const int64_t tiles = ((M + c.bm - 1) / c.bm) * n_tiles_of(false) * 2;
        if (tiles > units_of(false)) continue;
        const double cost = 1.15 * 128.0 * c.bm / c.eff / 2.0;
        if (cost < best - 1e-9) {
          best = cost;
          p.pair = false;
          p.bm = c.bm;
          long_k_split = 2;
        }
      }
    }
  }
  p.n_tiles = n_tiles_of(p.pair);
  const int units = units_of(p.pair);
  p.m_tiles = static_cast<int>((M + p.bm - 1) / p.bm);
  const int base_tiles = p.m_tiles * p.n_tiles;
  int s = 1;
  const int os = g_override_splits.load();
  if (os > 0) {
    s = os;
  } else if (long_k_split > 0) {
    s = long_k_split;
  } else if (allow_split && !p.twophase && base_tiles * 2 <= units && KB >= 8) {
    s = std::min(std::min(units / base_tiles, KB / 4), 16);
    // a caller with bounded scratch gets the most splits whose partial sums
    // fit it (an unsplit plan needs none, so an automatic plan always fits)
    if (max_split_ws != SIZE_MAX) {
      const size_t per_split = static_cast<size_t>(M) * N * sizeof(float);
      s = static_cast<int>(std::min<size_t>(s, std::max<size_t>(1, max_split_ws / per_split)));
    }
  }
  s = (allow_split && !p.twophase) ? std::max(1, std::min(s, KB)) : 1;
  p.kb_per_split = (KB + s - 1) / s;
  p.splits = (KB + p.kb_per_split - 1) / p.kb_per_split;
  p.tiles = base_tiles * p.splits;
  p.grid = std::min(p.tiles, units);  // CTAs (1-CTA kernel) or pairs (pair kernel)
  p.ws = p.splits > 1 ? static_cast<size_t>(p.splits) * M * N * sizeof(float) : 0;
  if (p.twophase)  // the bf16 weight, then the weight groups' ready counters
    p.ws = twophase_counter_offset(N, K) + twophase_counter_bytes(p.n_tiles);
  return p;
}

template <int FMT, int BM, int VAR>
static int launch_gemm(DeviceInfo* d, const Plan& p, const CUtensorMap& mx, const CUtensorMap& mw,
                       const GemmArgs& a, cudaStream_t st) {
  using C = GemmCfg<FMT, BM>;
  auto kern = dq_gemm_kernel<FMT, BM, VAR>;
  const int bi = bm_index(BM);
  const int rc = once_per_device(d->smem_set[VAR][FMT][bi], [&] {
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes) ==
                   cudaSuccess
               ? static_cast<int>(DQ_OK)
               : static_cast<int>(DQ_ERR_LAUNCH);
  });
  if (rc != DQ_OK) return rc;
  kern<<<p.grid, C::kThreads, C::kSmemBytes, st>>>(mx, mw, a);
  return cudaGetLastError() == cudaSuccess ? DQ_OK : DQ_ERR_LAUNCH;
}

// One-time setup of a pair-kernel instantiation on this device: shared-memory
// opt-in and the number of two-CTA clusters that can be resident at once
// (cached in d->max_pairs; the persistent grid never exceeds it).
template <int FMT, int BM, int VAR>
static int pair_setup(DeviceInfo* d, cudaLaunchConfig_t& cfg) {
  using C = Gemm2Cfg<FMT, BM>;
  auto kern = dq_gemm2_kernel<FMT, BM, VAR>;
  const int bi = bm_index(BM);
  return once_per_device(d->smem_set2[VAR][FMT][bi], [&] {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes) !=
        cudaSuccess)
      return static_cast<int>(DQ_ERR_LAUNCH);
    int clusters = 0;
    cfg.gridDim = dim3(2 * std::max(1, d->sms / 2));
    if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess || clusters < 1)
      return static_cast<int>(DQ_ERR_LAUNCH);
    d->max_pairs[VAR][FMT][bi] = clusters;
    return static_cast<int>(DQ_OK);
  });
}

template <int FMT, int BM>
static cudaLaunchConfig_t pair_config(cudaLaunchAttribute* attr, cudaStream_t st) {
  using C = Gemm2Cfg<FMT, BM>;
  cudaLaunchConfig_t cfg = {};
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(C::kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

template <int FMT, int BM, int VAR>
static int launch_gemm2(DeviceInfo* d, const Plan& p, const CUtensorMap& mx, const CUtensorMap& mw,
                        const GemmArgs& a, cudaStream_t st) {
  auto kern = dq_gemm2_kernel<FMT, BM, VAR>;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pair_config<FMT, BM>(attr, st);
  const int rc = pair_setup<FMT, BM, VAR>(d, cfg);
  if (rc != DQ_OK) return rc;
  const int pairs = std::max(1, std::min(p.grid, d->max_pairs[VAR][FMT][bm_index(BM)]));
  cfg.gridDim = dim3(2 * pairs);
  if (cudaLaunchKernelEx(&cfg, kern, mx, mw, a) != cudaSuccess) return DQ_ERR_LAUNCH;
  return cudaGetLastError() == cudaSuccess ? DQ_OK : DQ_ERR_LAUNCH;
}

// Resident-cluster capacity of the pair kernel for (FMT, bm) on this device.
template <int FMT>
static int pair_capacity(DeviceInfo* d, int bm, int* pairs) {
  cudaLaunchAttribute attr[1];
  int rc = DQ_ERR_ARG;
  switch (bm) {
    case 64: { auto c = pair_config<FMT, 64>(attr, nullptr); rc = pair_setup<FMT, 64, 0>(d, c); break; }
    case 128: { auto c = pair_config<FMT, 128>(attr, nullptr); rc = pair_setup<FMT, 128, 0>(d, c); break; }
    case 192: { auto c = pair_config<FMT, 192>(attr, nullptr); rc = pair_setup<FMT, 192, 0>(d, c); break; }
    case 256: { auto c = pair_config<FMT, 256>(attr, nullptr); rc = pair_setup<FMT, 256, 0>(d, c); break; }
  }
  if (rc == DQ_OK) *pairs = d->max_pairs[0][FMT][bm_index(bm)];
  return rc;
}

template <int BM, int FMT>
static cudaLaunchConfig_t bf16_pair_config(cudaLaunchAttribute* attr, cudaStream_t st) {
  using C = Bf16PairCfg<BM, FMT>;
  cudaLaunchConfig_t cfg = {};
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(C::kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

// One-time setup of a bf16 pair GEMM instantiation: shared-memory opt-in and
// the resident-cluster capacity (cached in d->bf16_max_pairs).
template <int BM, int FMT, bool TP = false>
static int bf16_pair_setup(DeviceInfo* d) {
  using C = Bf16PairCfg<BM, FMT>;
  const int bi = bm_index(BM);
  return once_per_device(d->bf16_smem_set[TP][FMT + 1][bi], [&] {
    auto kern = bf16_gemm2_kernel<BM, FMT, TP>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes) !=
        cudaSuccess)
      return static_cast<int>(DQ_ERR_LAUNCH);
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = bf16_pair_config<BM, FMT>(attr, nullptr);
    cfg.gridDim = dim3(2 * std::max(1, d->sms / 2));
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess || clusters < 1)
      return static_cast<int>(DQ_ERR_LAUNCH);
    d->bf16_max_pairs[TP][FMT + 1][bi] = clusters;
    return static_cast<int>(DQ_OK);
  });
}

template <int FMT>
static int bf16_pair_capacity(DeviceInfo* d, int bm, int* pairs) {
  int rc = DQ_ERR_ARG;
  switch (bm) {
    case 64: rc = bf16_pair_setup<64, FMT>(d); break;
    case 128: rc = bf16_pair_setup<128, FMT>(d); break;
    case 192: rc = bf16_pair_setup<192, FMT>(d); break;
    case 256: rc = bf16_pair_setup<256, FMT>(d); break;
  }
  if (rc == DQ_OK) *pairs = d->bf16_max_pairs[0][FMT + 1][bm_index(bm)];
  return rc;
}

// FMT >= 0: the launch also decodes the weight (a.dq_*), its first weight
// group just wide enough that the first wave of pairs finds all its tiles
// there.  Every CTA must be resident at once (the producers wait for the
// decode warps of all CTAs): the grid never exceeds the occupancy-derived
// number of resident pairs.
template <int BM, int FMT, bool TP = false>
static int launch_bf16_gemm2(DeviceInfo* d, const Plan& p, const CUtensorMap& mx,
                             const CUtensorMap& ma, const GemmArgs& a, cudaStream_t st) {
  const int rc = bf16_pair_setup<BM, FMT, TP>(d);
  if (rc != DQ_OK) return rc;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = bf16_pair_config<BM, FMT>(attr, st);
  const int pairs = std::max(1, std::min(p.grid, d->bf16_max_pairs[TP][FMT + 1][bm_index(BM)]));
  cfg.gridDim = dim3(2 * pairs);
  GemmArgs g = a;
  if (FMT >= 0) {
    const int m_tiles = std::max(1, p.m_tiles);
    g.group0_n = std::min(a.group_n, std::max(1, (pairs + m_tiles - 1) / m_tiles));
  }
  if (cudaLaunchKernelEx(&cfg, bf16_gemm2_kernel<BM, FMT, TP>, mx, ma, g) != cudaSuccess)
    return DQ_ERR_LAUNCH;
  return cudaGetLastError() == cudaSuccess ? DQ_OK : DQ_ERR_LAUNCH;
}

template <int FMT, bool TP = false>
static int launch_bf16_gemm2_bm(DeviceInfo* d, const Plan& p, const CUtensorMap& mx,
                                const CUtensorMap& ma, const GemmArgs& a, cudaStream_t st) {
  switch (p.bm) {
    case 64: return launch_bf16_gemm2<64, FMT, TP>(d, p, mx, ma, a, st);
    case 128: return launch_bf16_gemm2<128, FMT, TP>(d, p, mx, ma, a, st);
    case 192: return launch_bf16_gemm2<192, FMT, TP>(d, p, mx, ma, a, st);
    case 256: return launch_bf16_gemm2<256, FMT, TP>(d, p, mx, ma, a, st);
  }
  return DQ_ERR_ARG;
}

template <int FMT, int VAR>
static int dispatch_gemm(DeviceInfo* d, const Plan& p, const CUtensorMap& mx, const CUtensorMap& mw,
                         const GemmArgs& a, cudaStream_t st) {
  if (p.pair) {
    switch (p.bm) {
      case 64: return launch_gemm2<FMT, 64, VAR>(d, p, mx, mw, a, st);
      case 128: return launch_gemm2<FMT, 128, VAR>(d, p, mx, mw, a, st);
      case 192: return launch_gemm2<FMT, 192, VAR>(d, p, mx, mw, a, st);
      case 256: return launch_gemm2<FMT, 256, VAR>(d, p, mx, mw, a, st);
    }
    return DQ_ERR_ARG;
  }
  switch (p.bm) {
    case 16: return launch_gemm<FMT, 16, VAR>(d, p, mx, mw, a, st);
    case 32: return launch_gemm<FMT, 32, VAR>(d, p, mx, mw, a, st);
    case 64: return launch_gemm<FMT, 64, VAR>(d, p, mx, mw, a, st);
    case 128: return launch_gemm<FMT, 128, VAR>(d, p, mx, mw, a, st);
    case 192: return launch_gemm<FMT, 192, VAR>(d, p, mx, mw, a, st);
    case 256: return launch_gemm<FMT, 256, VAR>(d, p, mx, mw, a, st);
  }
  return DQ_ERR_ARG;
}

static inline bool aligned(const void* p, uintptr_t a) {
  return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0;
}

static int grid_for(int64_t work, int threads, int sms) {
  int64_t g = (work + threads - 1) / threads;
  g = std::min<int64_t>(g, static_cast<int64_t>(sms) * 16);
  return static_cast<int>(std::max<int64_t>(g, 1));
}

// Column-parallel call: this rank's N columns go to column rank * N of every
// rank's y [M, N * world].
struct TpOpts {
  int rank, world;
  void* const* y_ranks;
  unsigned int* const* flag_ranks;
  unsigned int* counter;
  unsigned int epoch;
  void* y_mc;  // multicast address of the call's y (all ranks' y buffers), or nullptr
};

static constexpr unsigned long long kTpWaitNs = 5000000000ull;  // 5 s

// The small-M kernel: one CTA per 16 * R16 weight rows, MT 8-token tiles.
template <int FMT, int MT, int R16, bool SBF>
static int launch_smallm_kern(DeviceInfo* d, const void* x, const uint8_t* w, const void* absmax,
                              float scale, const void* bias, void* y, int64_t M, int64_t N, int64_t K,
                              int act, int64_t ldy, cudaStream_t st) {
  using C = SmallMCfg<FMT, MT, R16>;
  auto kern = smallm_kernel<FMT, MT, R16, SBF>;
  const int rc = once_per_device(d->smallm_set[SBF ? 2 : FMT][MT - 1][R16 == 4 ? 2 : R16 - 1], [&] {
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes) ==
                   cudaSuccess
               ? static_cast<int>(DQ_OK)
               : static_cast<int>(DQ_ERR_LAUNCH);
  });
  if (rc != DQ_OK) return rc;
  const int grid = static_cast<int>((N + 16 * R16 - 1) / (16 * R16));
  kern<<<grid, C::kThreads, C::kSmemBytes, st>>>(
      static_cast<const __nv_bfloat16*>(x), w, absmax, scale,
      static_cast<const __nv_bfloat16*>(bias), static_cast<__nv_bfloat16*>(y),
      static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), act, ldy);
  return cudaGetLastError() == cudaSuccess ? DQ_OK : DQ_ERR_LAUNCH;
}

template <int FMT, int MT, int R16>
static int launch_smallm_cfg(DeviceInfo* d, const Plan& p, const void* x, const uint8_t* w,
                             const void* absmax, int sbf, float scale, const void* bias, void* y,
                             int64_t M, int64_t N, int64_t K, int act, int64_t ldy, cudaStream_t st) {
  if constexpr (FMT == kFmtNF4) {
    if (sbf) return launch_smallm_kern<FMT, MT, R16, true>(d, x, w, absmax, scale, bias, y, M, N, K, act, ldy, st);
  }
  return launch_smallm_kern<FMT, MT, R16, false>(d, x, w, absmax, scale, bias, y, M, N, K, act, ldy, st);
}

template <int FMT, int MT>
static int launch_smallm(DeviceInfo* d, const Plan& p, const void* x, const uint8_t* w,
                         const void* absmax, int sbf, float scale, const void* bias, void* y, int64_t M,
                         int64_t N, int64_t K, int act, int64_t ldy, cudaStream_t st) {
  switch (smallm_rows(FMT, M, N, d->sms, act_is_gated(act))) {
    case 4:
      if constexpr (MT == 1)
        return launch_smallm_cfg<FMT, MT, 4>(d, p, x, w, absmax, sbf, scale, bias, y, M, N, K, act, ldy, st);
      break;
    case 2:
      return launch_smallm_cfg<FMT, MT, 2>(d, p, x, w, absmax, sbf, scale, bias, y, M, N, K, act, ldy, st);
  }
  return launch_smallm_cfg<FMT, MT, 1>(d, p, x, w, absmax, sbf, scale, bias, y, M, N, K, act, ldy, st);
}

// The TMA-ring small-M kernel: one CTA per 16 * R16 weight rows, one 8-token
// tile, CPS CTAs per SM.
template <int FMT, int R16, int CPS, int MT = 1>
static int launch_smallm2_cfg(DeviceInfo* d, const void* x, const uint8_t* w, const void* absmax,
                              float scale, const void* bias, void* y, int64_t M, int64_t N,
                              int64_t K, int act, int64_t ldy, cudaStream_t st) {
  using C = SmallM2Cfg<FMT, MT, R16, CPS>;
  auto kern = smallm2_kernel<FMT, MT, R16, CPS>;
  std::atomic<int>& set_flag = MT == 2 ? d->smallm2_mt2_set[FMT]
                                       : d->smallm2_set[FMT][CPS - 2][R16 == 4 ? 2 : R16 - 1];
  const int rc = once_per_device(set_flag, [&] {
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes) ==
                   cudaSuccess
               ? static_cast<int>(DQ_OK)
               : static_cast<int>(DQ_ERR_LAUNCH);
  });
  if (rc != DQ_OK) return rc;
  CUtensorMap mw, ma;
  const uint64_t wrow = FMT == kFmtNF4 ? K / 2 : K;
  if (!make_map_2d(&mw, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, wrow, N, wrow, 128, C::kRows,
                   CU_TENSOR_MAP_SWIZZLE_128B))
    return DQ_ERR_CUDA;
  if constexpr (FMT == kFmtNF4) {
    if (!make_map_2d(&ma, absmax, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, K / 64, N, (K / 64) * 4,
                     C::kAbsPerRow, C::kRows, CU_TENSOR_MAP_SWIZZLE_NONE))
      return DQ_ERR_CUDA;
  } else {
    ma = mw;  // unused
  }
  CUtensorMap mx = mw;  // unused with one token tile
  if constexpr (MT == 2) {
    if (!make_map_2d(&mx, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, K, M, K * 2, 64, 16,
                     CU_TENSOR_MAP_SWIZZLE_128B))
      return DQ_ERR_CUDA;
  }
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>((N + C::kRows - 1) / C::kRows));
  cfg.blockDim = dim3(C::kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, mw, ma, mx, static_cast<const __nv_bfloat16*>(x), scale,
                         static_cast<const __nv_bfloat16*>(bias), static_cast<__nv_bfloat16*>(y),
                         static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), act,
                         ldy) != cudaSuccess)
    return DQ_ERR_LAUNCH;
  return cudaGetLastError() == cudaSuccess ? DQ_OK : DQ_ERR_LAUNCH;
}

template <int FMT, int CPS>
static int launch_smallm2_r(DeviceInfo* d, int r16, const void* x, const uint8_t* w, const void* absmax,
                            float scale, const void* bias, void* y, int64_t M, int64_t N, int64_t K,
                            int act, int64_t ldy, cudaStream_t st) {
  switch (r16) {
    case 4: return launch_smallm2_cfg<FMT, 4, CPS>(d, x, w, absmax, scale, bias, y, M, N, K, act, ldy, st);
    case 2: return launch_smallm2_cfg<FMT, 2, CPS>(d, x, w, absmax, scale, bias, y, M, N, K, act, ldy, st);
  }
  return launch_smallm2_cfg<FMT, 1, CPS>(d, x, w, absmax, scale, bias, y, M, N, K, act, ldy, st);
}

template <int FMT>
static int launch_smallm2(DeviceInfo* d, const Plan& p, const void* x, const uint8_t* w,
                          const void* absmax, float scale, const void* bias, void* y, int64_t M,
                          int64_t N, int64_t K, int act, int64_t ldy, cudaStream_t st) {
  if (M > 8)
    return launch_smallm2_cfg<FMT, 4, 2, 2>(d, x, w, absmax, scale, bias, y, M, N, K, act, ldy, st);
  return p.cps == 3 ? launch_smallm2_r<FMT, 3>(d, p.r16, x, w, absmax, scale, bias, y, M, N, K, act, ldy, st)
                    : launch_smallm2_r<FMT, 2>(d, p.r16, x, w, absmax, scale, bias, y, M, N, K, act, ldy, st);
}

static int linear_impl(int fmt, const void* x, int64_t M, int64_t K, const uint8_t* w,
                       const void* absmax, float scale, const void* bias, int64_t N, void* y,
                       void* ws, size_t ws_bytes, cudaStream_t st, const TpOpts* tp = nullptr,
                       bool allow_twophase = true, int act = kActNone, int64_t ldy = 0,
                       size_t max_split_ws = SIZE_MAX, int scale_dtype = DQ_DTYPE_F32) {
  if (act < kActNone || act > kActGeGluTanh) return DQ_ERR_ARG;
  const bool gated = act_is_gated(act);
  // a gated activation takes 32-row groups of the gated row order and writes
  // N / 2 columns; the column-parallel path has no gated epilogue
  if (gated && tp != nullptr) return DQ_ERR_ARG;
  if (gated && (N <= 0 || N % 32 != 0)) return DQ_ERR_SHAPE;
  const int64_t n_out = gated ? N / 2 : N;
  // y row stride (elements): the output width unless the caller writes into a
  // wider buffer
  if (ldy == 0) ldy = n_out;
  if (ldy < n_out || ldy > INT32_MAX || (tp != nullptr && ldy != N)) return DQ_ERR_SHAPE;
  // NF4 blocks of 64 must lie inside a weight row; fp8 needs only 16-byte
  // row strides for TMA (the ragged last k-block is zero-filled).
  if (M < 0 || N <= 0 || K <= 0 || (K % (fmt == kFmtNF4 ? 64 : 16)) != 0) return DQ_ERR_SHAPE;
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return DQ_ERR_SHAPE;
  if (M == 0) return DQ_OK;
  if (scale_dtype != DQ_DTYPE_F32 && scale_dtype != DQ_DTYPE_BF16) return DQ_ERR_ARG;
  const int sbf = (fmt == kFmtNF4 && scale_dtype == DQ_DTYPE_BF16) ? 1 : 0;
  if (x == nullptr || w == nullptr || y == nullptr || (fmt == kFmtNF4 && absmax == nullptr))
    return DQ_ERR_ARG;
  if (!aligned(x, 16) || !aligned(w, 16) || !aligned(absmax, sbf ? 2 : 4) || !aligned(bias, 2) ||
      !aligned(y, 2))
    return DQ_ERR_ALIGN;
  DeviceInfo* d = nullptr;
  int rc = current_device(&d);
  if (rc != DQ_OK) return rc;
  // the column-parallel path takes the two-phase plan only when its caller
  // lends a workspace (the dq_tp_linear_*_ws entry points)
  const Plan p = make_plan(fmt, M, N, K, d->sms, tp == nullptr,
                           allow_twophase && (tp == nullptr || ws != nullptr), tp == nullptr,
                           max_split_ws, gated);
  if (max_split_ws != SIZE_MAX && p.ws > max_split_ws) return DQ_ERR_SCRATCH_LIMIT;
  if (p.ws > 0 && (ws == nullptr || ws_bytes < p.ws || !aligned(ws, 16))) return DQ_ERR_WORKSPACE;

  if (p.smallm && p.ring && (fmt != kFmtNF4 || (!sbf && aligned(absmax, 16)))) {
    return fmt == kFmtNF4
               ? launch_smallm2<kFmtNF4>(d, p, x, w, absmax, scale, bias, y, M, N, K, act, ldy, st)
               : launch_smallm2<kFmtFP8>(d, p, x, w, absmax, scale, bias, y, M, N, K, act, ldy, st);
  }
  // (a ring plan whose NF4 scales are bf16 or not 16-byte aligned falls
  // through to the register-stream kernel, which picks its own row groups)
  if (p.smallm) {
    if (fmt == kFmtNF4)
      return p.bm <= 8 ? launch_smallm<kFmtNF4, 1>(d, p, x, w, absmax, sbf, scale, bias, y, M, N, K, act, ldy, st)
                       : launch_smallm<kFmtNF4, 2>(d, p, x, w, absmax, sbf, scale, bias, y, M, N, K, act, ldy, st);
    return p.bm <= 8 ? launch_smallm<kFmtFP8, 1>(d, p, x, w, absmax, sbf, scale, bias, y, M, N, K, act, ldy, st)
                     : launch_smallm<kFmtFP8, 2>(d, p, x, w, absmax, sbf, scale, bias, y, M, N, K, act, ldy, st);
  }

  if (p.twophase) {
    // The weight is dequantized once into the bf16 scratch [N, K] and read
    // by a bf16 x bf16 pair GEMM.  Normally the GEMM launch decodes it
    // itself, group by group under the MMAs (the ready counters after the
    // scratch start at zero); pair mode 4 runs the decode as its own launch
    // first.
    const bool separate = tp == nullptr && g_override_pair.load() == 4;
    unsigned int* ready =
        reinterpret_cast<unsigned int*>(static_cast<uint8_t*>(ws) + twophase_counter_offset(N, K));
    if (separate) {
      const int64_t n_elems = N * K;
      if (fmt == kFmtNF4) {
        dequant_nf4_kernel<<<decode_grid(n_elems / 32, d->sms), 256, 0, st>>>(
            reinterpret_cast<const uint4*>(w), absmax, static_cast<uint4*>(ws), n_elems / 32, sbf);
      } else {
        dequant_fp8_kernel<<<decode_grid(n_elems / 16 + 1, d->sms), 256, 0, st>>>(
            w, scale, static_cast<__nv_bfloat16*>(ws), n_elems);
      }
      if (cudaGetLastError() != cudaSuccess) return DQ_ERR_LAUNCH;
    } else if (cudaMemsetAsync(ready, 0, twophase_counter_bytes(p.n_tiles), st) != cudaSuccess) {
      return DQ_ERR_CUDA;
    }
    CUtensorMap mx2, ma;
    if (!make_map_2d(&mx2, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, K, M, K * 2, 64, p.bm / 2,
                     CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_map_2d(&ma, ws, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, K, N, K * 2, 64, 128,
                     CU_TENSOR_MAP_SWIZZLE_128B))
      return DQ_ERR_CUDA;
    GemmArgs g = {};
    g.absmax = static_cast<const float*>(absmax);
    g.scale_bf16 = sbf;
    g.bias = static_cast<const __nv_bfloat16*>(bias);
    g.out = nullptr;
    g.M = static_cast<int>(M);
    g.N = static_cast<int>(N);
    g.K = static_cast<int>(K);
    g.num_n_tiles = p.n_tiles;
    g.tile_n = 256;
    g.num_tiles = p.tiles;
    g.splits = 1;
    g.kb_per_split = p.kb_per_split;
    g.group_n = kTwoPhaseGroupN;  // the bf16 weight no longer fits L2 beside X and Y
    g.group0_n = 0;
    g.act = act;
    g.fp8_scale = scale;
    g.dq_w = w;
    g.dq_out = static_cast<__nv_bfloat16*>(ws);
    g.dq_ready = ready;
    for (int r = 0; r < kMaxRanks; ++r) {
      g.outs[r] = nullptr;
      g.tp_flags[r] = nullptr;
    }
    g.outs[0] = y;
    g.n_out = 1;
    g.ldy = static_cast<int>(ldy);
    g.col0 = 0;
    g.vec_ok = (n_out % 8 == 0) && (ldy % 8 == 0) && aligned(y, 16);
    g.tp_counter = nullptr;
    g.tp_rank = 0;
    g.tp_epoch = 0;
    if (tp != nullptr) {
      // every rank's y [M, N * world] at column N * rank, then the flags
      g.n_out = tp->world;
      g.ldy = static_cast<int>(N * tp->world);
      g.col0 = static_cast<int>(N * tp->rank);
      g.vec_ok = (N % 8 == 0);
      for (int r = 0; r < tp->world; ++r) {
        g.outs[r] = tp->y_ranks[r];
        g.tp_flags[r] = tp->flag_ranks[r];
        g.vec_ok = g.vec_ok && aligned(tp->y_ranks[r], 16);
      }
      g.tp_counter = tp->counter;
      g.tp_rank = tp->rank;
      g.tp_epoch = tp->epoch;
      g.out_mc = g.vec_ok && aligned(tp->y_mc, 16) ? tp->y_mc : nullptr;
      rc = fmt == kFmtNF4 ? launch_bf16_gemm2_bm<kFmtNF4, true>(d, p, mx2, ma, g, st)
                          : launch_bf16_gemm2_bm<kFmtFP8, true>(d, p, mx2, ma, g, st);
      if (rc != DQ_OK) return rc;
      tp_wait_kernel<<<1, 32, 0, st>>>(tp->flag_ranks[tp->rank], tp->world, tp->epoch, kTpWaitNs);
      return cudaGetLastError() == cudaSuccess ? DQ_OK : DQ_ERR_LAUNCH;
    }
    if (separate) return launch_bf16_gemm2_bm<-1>(d, p, mx2, ma, g, st);
    return fmt == kFmtNF4 ? launch_bf16_gemm2_bm<kFmtNF4>(d, p, mx2, ma, g, st)
                          : launch_bf16_gemm2_bm<kFmtFP8>(d, p, mx2, ma, g, st);
  }

  CUtensorMap mx, mw;
  if (!make_map_2d(&mx, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, K, M, K * 2, 64,
                   p.pair ? p.bm / 2 : p.bm, CU_TENSOR_MAP_SWIZZLE_128B))
    return DQ_ERR_CUDA;
  const uint64_t wrow = fmt == kFmtNF4 ? K / 2 : K;
  if (!make_map_2d(&mw, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, wrow, N, wrow,
                   fmt == kFmtNF4 ? 32 : 64, 128,
                   fmt == kFmtNF4 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B))
    return DQ_ERR_CUDA;

  GemmArgs a = {};
  a.absmax = static_cast<const float*>(absmax);
  a.scale_bf16 = sbf;
  a.bias = static_cast<const __nv_bfloat16*>(bias);
  a.M = static_cast<int>(M);
  a.N = static_cast<int>(N);
  a.K = static_cast<int>(K);
  a.num_n_tiles = p.n_tiles;
  a.tile_n = p.pair ? 256 : 128;
  a.num_tiles = p.tiles;
  a.splits = p.splits;
  a.kb_per_split = p.kb_per_split;
  a.group_n = 0;
  a.group0_n = 0;
  a.dq_w = nullptr;
  a.dq_out = nullptr;
  a.dq_ready = nullptr;
  a.act = act;
  a.fp8_scale = scale;
  for (int r = 0; r < kMaxRanks; ++r) {
    a.outs[r] = nullptr;
    a.tp_flags[r] = nullptr;
  }
  a.tp_counter = nullptr;
  a.tp_rank = 0;
  a.tp_epoch = 0;
  a.out = nullptr;
  if (p.splits > 1) {
    a.out = ws;
    a.vec_ok = (N % 4 == 0) && aligned(ws, 16);
    a.n_out = 0;
    a.ldy = static_cast<int>(N);
    a.col0 = 0;
  } else if (tp == nullptr) {
    a.outs[0] = y;
    a.n_out = 1;
    a.ldy = static_cast<int>(ldy);
    a.col0 = 0;
    a.vec_ok = (n_out % 8 == 0) && (ldy % 8 == 0) && aligned(y, 16);
  } else {
    a.n_out = tp->world;
    a.ldy = static_cast<int>(N * tp->world);
    a.col0 = static_cast<int>(N * tp->rank);
    a.vec_ok = (N % 8 == 0);
    for (int r = 0; r < tp->world; ++r) {
      a.outs[r] = tp->y_ranks[r];
      a.tp_flags[r] = tp->flag_ranks[r];
      a.vec_ok = a.vec_ok && aligned(tp->y_ranks[r], 16);
    }
    a.tp_counter = tp->counter;
    a.tp_rank = tp->rank;
    a.tp_epoch = tp->epoch;
    a.out_mc = a.vec_ok && aligned(tp->y_mc, 16) ? tp->y_mc : nullptr;
  }
  if (tp != nullptr) {
    rc = fmt == kFmtNF4 ? dispatch_gemm<kFmtNF4, 1>(d, p, mx, mw, a, st)
                        : dispatch_gemm<kFmtFP8, 1>(d, p, mx, mw, a, st);
  } else if (gated && p.splits == 1) {
    rc = fmt == kFmtNF4 ? dispatch_gemm<kFmtNF4, 2>(d, p, mx, mw, a, st)
                        : dispatch_gemm<kFmtFP8, 2>(d, p, mx, mw, a, st);
  } else {
    // (split-K partials are written raw; the reduce kernel applies the gate)
    rc = fmt == kFmtNF4 ? dispatch_gemm<kFmtNF4, 0>(d, p, mx, mw, a, st)
                        : dispatch_gemm<kFmtFP8, 0>(d, p, mx, mw, a, st);
  }
  if (rc != DQ_OK) return rc;
  if (p.splits > 1) {
    const int64_t total = M * n_out;
    splitk_reduce_kernel<<<grid_for(total, 256, d->sms), 256, 0, st>>>(
        static_cast<const float*>(ws), p.splits, a.M, a.N, a.bias,
        static_cast<__nv_bfloat16*>(y), a.act, ldy);
    if (cudaGetLastError() != cudaSuccess) return DQ_ERR_LAUNCH;
  }
  if (tp != nullptr) {
    tp_wait_kernel<<<1, 32, 0, st>>>(tp->flag_ranks[tp->rank], tp->world, tp->epoch, kTpWaitNs);
    if (cudaGetLastError() != cudaSuccess) return DQ_ERR_LAUNCH;
  }
  return DQ_OK;
}

static int tp_impl(int fmt, const void* x, int64_t M, int64_t K, const uint8_t* w,
                   const float* absmax, float scale, const void* bias, int64_t N, int rank,
                   int world, void* const* y_ranks, unsigned int* const* flag_ranks,
                   unsigned int* counter, unsigned int epoch, cudaStream_t st,
                   void* ws = nullptr, size_t ws_bytes = 0, void* y_mc = nullptr) {
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world) return DQ_ERR_ARG;
  if (y_ranks == nullptr || flag_ranks == nullptr || counter == nullptr) return DQ_ERR_ARG;
  if (N <= 0 || (N % world) != 0) return DQ_ERR_SHAPE;
  for (int r = 0; r < world; ++r) {
    if (y_ranks[r] == nullptr || flag_ranks[r] == nullptr) return DQ_ERR_ARG;
    if (!aligned(y_ranks[r], 2) || !aligned(flag_ranks[r], 4)) return DQ_ERR_ALIGN;
  }
  if (!aligned(counter, 4)) return DQ_ERR_ALIGN;
  if (M == 0) return DQ_OK;
  TpOpts tp{rank, world, y_ranks, flag_ranks, counter, epoch, y_mc};
  return linear_impl(fmt, x, M, K, w, absmax, scale, bias, N / world, y_ranks[rank], ws, ws_bytes,
                     st, &tp);
}

}  // namespace dq

using namespace dq;

template <int NPT>
static void launch_adaln(const void* x, int64_t ld_x, int64_t T, int S, int D, const void* scale,
                         const void* shift, int64_t ld_mod, float eps, void* out, int64_t ld_out,
                         cudaStream_t st) {
  adaln_modulate_kernel<NPT><<<static_cast<int>(T), 256, 0, st>>>(
      static_cast<const __nv_bfloat16*>(x), ld_x, S, D, static_cast<const __nv_bfloat16*>(scale),
      static_cast<const __nv_bfloat16*>(shift), ld_mod, eps, static_cast<__nv_bfloat16*>(out),
      ld_out);
}

extern "C" {

const char* dq_version(void) { return DQ_VERSION_STRING; }

int dq_abi_version(void) { return 2; }

const char* dq_status_string(int s) {
  switch (s) {
    case DQ_OK: return "ok";
    case DQ_ERR_SHAPE: return "bad shape (sizes must be positive, K and lengths multiples of 64)";
    case DQ_ERR_ALIGN: return "operand not 16-byte aligned";
    case DQ_ERR_ARCH: return "current device is not sm_100 (B200)";
    case DQ_ERR_LAUNCH: return "kernel launch failed";
    case DQ_ERR_TIMEOUT: return "a kernel wait timed out";
    case DQ_ERR_WORKSPACE: return "workspace missing or too small";
    case DQ_ERR_ARG: return "null operand or unknown enum";
    case DQ_ERR_CUDA: return "CUDA runtime error";
    case DQ_ERR_SCRATCH_LIMIT:
      return "shape needs more split-K scratch than the allocation-free entry point holds (8 MiB)";
  }
  return "unknown status";
}

int dq_quantize_nf4(const void* w, int w_dtype, int64_t n_elems, uint8_t* packed, float* absmax,
                    dq_stream_t stream) {
  if (n_elems < 0 || (n_elems % 64) != 0) return DQ_ERR_SHAPE;
  if (n_elems == 0) return DQ_OK;
  if (w == nullptr || packed == nullptr || absmax == nullptr) return DQ_ERR_ARG;
  if (w_dtype != DQ_DTYPE_F32 && w_dtype != DQ_DTYPE_BF16) return DQ_ERR_ARG;
  DeviceInfo* d = nullptr;
  int rc = current_device(&d);
  if (rc != DQ_OK) return rc;
  const int64_t nb = n_elems / 64;
  const int grid = grid_for(nb * 32, 256, d->sms);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (w_dtype == DQ_DTYPE_F32)
    quantize_nf4_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(w), packed, absmax, nb);
  else
    quantize_nf4_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(w),
                                                             packed, absmax, nb);
  return cudaGetLastError() == cudaSuccess ? DQ_OK : DQ_ERR_LAUNCH;
}

int dq_quantize_fp8(const void* w, int w_dtype, int64_t n_elems, uint8_t* w8, float* scale_out,
                    dq_stream_t stream) {
  if (n_elems <= 0) return DQ_ERR_SHAPE;
  if (w == nullptr || w8 == nullptr || scale_out == nullptr) return DQ_ERR_ARG;
  if (w_dtype != DQ_DTYPE_F32 && w_dtype != DQ_DTYPE_BF16) return DQ_ERR_ARG;
  if (!aligned(scale_out, 4)) return DQ_ERR_ALIGN;
  DeviceInfo* d = nullptr;
  int rc = current_device(&d);
  if (rc != DQ_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  unsigned int* bits = reinterpret_cast<unsigned int*>(scale_out);
  if (cudaMemsetAsync(bits, 0, sizeof(unsigned int), st) != cudaSuccess) return DQ_ERR_CUDA;
  const int grid = grid_for(n_elems, 256, d->sms);
  if (w_dtype == DQ_DTYPE_F32) {
    absmax_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(w), n_elems, bits);
    quantize_fp8_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(w), n_elems, bits, w8);
  } else {
    absmax_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(w), n_elems, bits);
    quantize_fp8_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(w),
                                                             n_elems, bits, w8);
  }
  finalize_fp8_scale_kernel<<<1, 1, 0, st>>>(bits);
  return cudaGetLastError() == cudaSuccess ? DQ_OK : DQ_ERR_LAUNCH;
}

int dq_dequant_nf4(const uint8_t* packed, const float* absmax, int64_t n_elems, void* out_bf16,
                   dq_stream_t stream) {
  if (n_elems < 0 || (n_elems % 64) != 0) return DQ_ERR_SHAPE;
  if (n_elems == 0) return DQ_OK;
  if (packed == nullptr || absmax == nullptr || out_bf16 == nullptr) return DQ_ERR_ARG;
  if (!aligned(packed, 16) || !aligned(out_bf16, 16) || !aligned(absmax, 4)) return DQ_ERR_ALIGN;
  DeviceInfo* d = nullptr;
  int rc = current_device(&d);
  if (rc != DQ_OK) return rc;
  const int64_t chunks = n_elems / 32;
  dequant_nf4_kernel<<<decode_grid(chunks, d->sms), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint4*>(packed), absmax, static_cast<uint4*>(out_bf16), chunks, 0);
  return cudaGetLastError() == cudaSuccess ? DQ_OK : DQ_ERR_LAUNCH;
}

int dq_dequant_fp8(const uint8_t* w8, float scale, int64_t n_elems, void* out_bf16,
                   dq_stream_t stream) {
  if (n_elems < 0) return DQ_ERR_SHAPE;
  if (n_elems == 0) return DQ_OK;
  if (w8 == nullptr || out_bf16 == nullptr) return DQ_ERR_ARG;
  if (!aligned(w8, 16) || !aligned(out_bf16, 16)) return DQ_ERR_ALIGN;
  DeviceInfo* d = nullptr;
  int rc = current_device(&d);
  if (rc != DQ_OK) return rc;
  dequant_fp8_kernel<<<decode_grid(n_elems / 16 + 1, d->sms), 256, 0,
                       static_cast<cudaStream_t>(stream)>>>(w8, scale,
                                                            static_cast<__nv_bfloat16*>(out_bf16), n_elems);
  return cudaGetLastError() == cudaSuccess ? DQ_OK : DQ_ERR_LAUNCH;
}

size_t dq_workspace_size(int64_t M, int64_t N, int64_t K, int fmt) {
  if (M <= 0 || N <= 0 || K <= 0 || (K % (fmt == DQ_FMT_NF4 ? 64 : 16)) != 0) return 0;
  DeviceInfo* d = nullptr;
  if (current_device(&d) != DQ_OK || d == nullptr) return 0;
  return make_plan(fmt, M, N, K, d->sms).ws;
}

int dq_linear_nf4_ld(const void* x, int64_t M, int64_t K, const uint8_t* packed,
                     const float* absmax, const void* bias, int64_t N, int act, void* y,
                     int64_t ldy, void* workspace, size_t workspace_bytes, dq_stream_t stream) {
  if (ldy <= 0) return DQ_ERR_SHAPE;  // linear_impl refuses strides below the output width
  return linear_impl(kFmtNF4, x, M, K, packed, absmax, 0.f, bias, N, y, workspace, workspace_bytes,
                     static_cast<cudaStream_t>(stream), nullptr, true, act, ldy);
}

int dq_linear_nf4_scaled(const void* x, int64_t M, int64_t K, const uint8_t* packed,
                         const void* absmax, int scale_dtype, const void* bias, int64_t N, int act,
                         void* y, int64_t ldy, void* workspace, size_t workspace_bytes,
                         dq_stream_t stream) {
  if (ldy < 0) return DQ_ERR_SHAPE;  // 0: the output width
  return linear_impl(kFmtNF4, x, M, K, packed, absmax, 0.f, bias, N, y, workspace, workspace_bytes,
                     static_cast<cudaStream_t>(stream), nullptr, true, act, ldy, SIZE_MAX,
                     scale_dtype);
}

int dq_dequant_nf4_scaled(const uint8_t* packed, const void* absmax, int scale_dtype,
                          int64_t n_elems, void* out_bf16, dq_stream_t stream) {
  if (scale_dtype != DQ_DTYPE_F32 && scale_dtype != DQ_DTYPE_BF16) return DQ_ERR_ARG;
  const int sbf = scale_dtype == DQ_DTYPE_BF16 ? 1 : 0;
  if (n_elems < 0 || (n_elems % 64) != 0) return DQ_ERR_SHAPE;
  if (n_elems == 0) return DQ_OK;
  if (packed == nullptr || absmax == nullptr || out_bf16 == nullptr) return DQ_ERR_ARG;
  if (!aligned(packed, 16) || !aligned(out_bf16, 16) || !aligned(absmax, sbf ? 2 : 4)) return DQ_ERR_ALIGN;
  DeviceInfo* d = nullptr;
  int rc = current_device(&d);
  if (rc != DQ_OK) return rc;
  const int64_t chunks = n_elems / 32;
  dequant_nf4_kernel<<<decode_grid(chunks, d->sms), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint4*>(packed), absmax, static_cast<uint4*>(out_bf16), chunks, sbf);
  return cudaGetLastError() == cudaSuccess ? DQ_OK : DQ_ERR_LAUNCH;
}

int dq_linear_fp8_ld(const void* x, int64_t M, int64_t K, const uint8_t* w8, float scale,
                     const void* bias, int64_t N, int act, void* y, int64_t ldy, void* workspace,
                     size_t workspace_bytes, dq_stream_t stream) {
  if (ldy <= 0) return DQ_ERR_SHAPE;  // linear_impl refuses strides below the output width
  return linear_impl(kFmtFP8, x, M, K, w8, nullptr, scale, bias, N, y, workspace, workspace_bytes,
                     static_cast<cudaStream_t>(stream), nullptr, true, act, ldy);
}

int dq_linear_nf4_ex(const void* x, int64_t M, int64_t K, const uint8_t* packed,
                     const float* absmax, const void* bias, int64_t N, int act, void* y,
                     void* workspace, size_t workspace_bytes, dq_stream_t stream) {
  return linear_impl(kFmtNF4, x, M, K, packed, absmax, 0.f, bias, N, y, workspace, workspace_bytes,
                     static_cast<cudaStream_t>(stream), nullptr, true, act);
}

int dq_linear_fp8_ex(const void* x, int64_t M, int64_t K, const uint8_t* w8, float scale,
                     const void* bias, int64_t N, int act, void* y, void* workspace,
                     size_t workspace_bytes, dq_stream_t stream) {
  return linear_impl(kFmtFP8, x, M, K, w8, nullptr, scale, bias, N, y, workspace, workspace_bytes,
                     static_cast<cudaStream_t>(stream), nullptr, true, act);
}

int dq_plan_info(int64_t M, int64_t N, int64_t K, int fmt, int* pair, int* bm, int* splits,
                 int* grid) {
  if (pair == nullptr || bm == nullptr || splits == nullptr || grid == nullptr) return DQ_ERR_ARG;
  if (M <= 0 || N <= 0 || K <= 0 || (fmt != DQ_FMT_NF4 && fmt != DQ_FMT_FP8) ||
      (K % (fmt == DQ_FMT_NF4 ? 64 : 16)) != 0)
    return DQ_ERR_SHAPE;
  DeviceInfo* d = nullptr;
  const int rc = current_device(&d);
  if (rc != DQ_OK) return rc;
  const Plan p = make_plan(fmt, M, N, K, d->sms);
  *pair = p.smallm ? (p.ring ? 4 : 3) : p.twophase ? 2 : (p.pair ? 1 : 0);
  *bm = p.bm;
  *splits = p.splits;
  *grid = p.grid;
  if (p.twophase) {
    int cap = 0;
    const int prc = g_override_pair.load() == 4 ? bf16_pair_capacity<-1>(d, p.bm, &cap)
                    : fmt == DQ_FMT_NF4         ? bf16_pair_capacity<kFmtNF4>(d, p.bm, &cap)
                                                : bf16_pair_capacity<kFmtFP8>(d, p.bm, &cap);
    if (prc != DQ_OK) return prc;
    *grid = 2 * std::max(1, std::min(p.grid, cap));
  } else if (p.pair) {
    int cap = 0;
    const int prc = fmt == DQ_FMT_NF4 ? pair_capacity<kFmtNF4>(d, p.bm, &cap)
                                      : pair_capacity<kFmtFP8>(d, p.bm, &cap);
    if (prc != DQ_OK) return prc;
    *grid = 2 * std::max(1, std::min(p.grid, cap));
  }
  return DQ_OK;
}

int dq_linear_nf4(const void* x, int64_t M, int64_t K, const uint8_t* packed, const float* absmax,
                  const void* bias, int64_t N, void* y, void* workspace, size_t workspace_bytes,
                  dq_stream_t stream) {
  return linear_impl(kFmtNF4, x, M, K, packed, absmax, 0.f, bias, N, y, workspace, workspace_bytes,
                     static_cast<cudaStream_t>(stream));
}

int dq_linear_fp8(const void* x, int64_t M, int64_t K, const uint8_t* w8, float scale,
                  const void* bias, int64_t N, void* y, void* workspace, size_t workspace_bytes,
                  dq_stream_t stream) {
  return linear_impl(kFmtFP8, x, M, K, w8, nullptr, scale, bias, N, y, workspace, workspace_bytes,
                     static_cast<cudaStream_t>(stream));
}

}  // extern "C"

namespace dq {
// Built-in split-K scratch of dq_linear_nf4_noalloc.  In host code the symbol
// is only a stand-in: kernels receive the device address that
// cudaGetSymbolAddress returns for the current device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[DQ_NOALLOC_SCRATCH_BYTES];
static std::atomic<void*> g_noalloc_addr[kMaxDevices];
static std::mutex g_noalloc_mu;
}  // namespace dq

extern "C" {

int dq_linear_nf4_noalloc(const void* x, int64_t M, int64_t K, const uint8_t* packed,
                          const float* absmax, const void* bias, int64_t N, void* y,
                          dq_stream_t stream) {
  // Arguments are validated by linear_impl, in the same order as for
  // dq_linear_nf4; a plan whose partial sums exceed the built-in array (only a
  // forced split count) returns DQ_ERR_SCRATCH_LIMIT there, before any launch.
  DeviceInfo* d = nullptr;
  int rc = current_device(&d);
  if (rc != DQ_OK) return rc;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return DQ_ERR_CUDA;
  void* scratch = g_noalloc_addr[dev].load();
  if (scratch == nullptr) {
    // First call on this device (with it current): look up the array's
    // device address once.
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    scratch = g_noalloc_addr[dev].load();
    if (scratch == nullptr) {
      if (cudaGetSymbolAddress(&scratch, g_noalloc_scratch) != cudaSuccess || scratch == nullptr)
        return DQ_ERR_CUDA;
      g_noalloc_addr[dev].store(scratch);
    }
  }
  return linear_impl(kFmtNF4, x, M, K, packed, absmax, 0.f, bias, N, y, scratch,
                     DQ_NOALLOC_SCRATCH_BYTES, static_cast<cudaStream_t>(stream), nullptr, false,
                     kActNone, 0, DQ_NOALLOC_SCRATCH_BYTES);
}

int dq_tp_buffer_alloc(size_t bytes, void** ptr) {
  if (ptr == nullptr || bytes == 0) return DQ_ERR_ARG;
  *ptr = nullptr;
  if (cudaMalloc(ptr, bytes) != cudaSuccess) return DQ_ERR_CUDA;
  if (cudaMemset(*ptr, 0, bytes) != cudaSuccess) return DQ_ERR_CUDA;
  return DQ_OK;
}

int dq_tp_buffer_free(void* ptr) {
  if (ptr == nullptr) return DQ_OK;
  return cudaFree(ptr) == cudaSuccess ? DQ_OK : DQ_ERR_CUDA;
}

int dq_ipc_handle(const void* ptr, void* handle_out) {
  static_assert(sizeof(cudaIpcMemHandle_t) == DQ_IPC_HANDLE_BYTES, "IPC handle size");
  if (ptr == nullptr || handle_out == nullptr) return DQ_ERR_ARG;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)) != cudaSuccess) return DQ_ERR_CUDA;
  std::memcpy(handle_out, &h, sizeof(h));
  return DQ_OK;
}

int dq_ipc_open(const void* handle, void** ptr) {
  if (handle == nullptr || ptr == nullptr) return DQ_ERR_ARG;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  *ptr = nullptr;
  if (cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
    return DQ_ERR_CUDA;
  return DQ_OK;
}

int dq_ipc_close(void* ptr) {
  if (ptr == nullptr) return DQ_OK;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? DQ_OK : DQ_ERR_CUDA;
}

int dq_tp_linear_nf4(const void* x, int64_t M, int64_t K, const uint8_t* packed_shard,
                     const float* absmax_shard, const void* bias_shard, int64_t N, int rank,
                     int world, void* const* y_ranks, unsigned int* const* flag_ranks,
                     unsigned int* counter, unsigned int epoch, dq_stream_t stream) {
  return tp_impl(kFmtNF4, x, M, K, packed_shard, absmax_shard, 0.f, bias_shard, N, rank, world,
                 y_ranks, flag_ranks, counter, epoch, static_cast<cudaStream_t>(stream));
}

int dq_tp_linear_fp8(const void* x, int64_t M, int64_t K, const uint8_t* w8_shard, float scale,
                     const void* bias_shard, int64_t N, int rank, int world, void* const* y_ranks,
                     unsigned int* const* flag_ranks, unsigned int* counter, unsigned int epoch,
                     dq_stream_t stream) {
  return tp_impl(kFmtFP8, x, M, K, w8_shard, nullptr, scale, bias_shard, N, rank, world, y_ranks,
                 flag_ranks, counter, epoch, static_cast<cudaStream_t>(stream));
}

int dq_tp_linear_nf4_ws(const void* x, int64_t M, int64_t K, const uint8_t* packed_shard,
                        const float* absmax_shard, const void* bias_shard, int64_t N, int rank,
                        int world, void* const* y_ranks, unsigned int* const* flag_ranks,
                        unsigned int* counter, unsigned int epoch, void* workspace,
                        size_t workspace_bytes, dq_stream_t stream) {
  if (workspace == nullptr) return DQ_ERR_WORKSPACE;
  return tp_impl(kFmtNF4, x, M, K, packed_shard, absmax_shard, 0.f, bias_shard, N, rank, world,
                 y_ranks, flag_ranks, counter, epoch, static_cast<cudaStream_t>(stream), workspace,
                 workspace_bytes);
}

int dq_tp_linear_fp8_ws(const void* x, int64_t M, int64_t K, const uint8_t* w8_shard, float scale,
                        const void* bias_shard, int64_t N, int rank, int world, void* const* y_ranks,
                        unsigned int* const* flag_ranks, unsigned int* counter, unsigned int epoch,
                        void* workspace, size_t workspace_bytes, dq_stream_t stream) {
  if (workspace == nullptr) return DQ_ERR_WORKSPACE;
  return tp_impl(kFmtFP8, x, M, K, w8_shard, nullptr, scale, bias_shard, N, rank, world, y_ranks,
                 flag_ranks, counter, epoch, static_cast<cudaStream_t>(stream), workspace,
                 workspace_bytes);
}

int dq_tp_linear_nf4_mc_ws(const void* x, int64_t M, int64_t K, const uint8_t* packed_shard,
                           const float* absmax_shard, const void* bias_shard, int64_t N, int rank,
                           int world, void* const* y_ranks, void* y_multicast,
                           unsigned int* const* flag_ranks, unsigned int* counter,
                           unsigned int epoch, void* workspace, size_t workspace_bytes,
                           dq_stream_t stream) {
  if (workspace == nullptr) return DQ_ERR_WORKSPACE;
  if (y_multicast == nullptr) return DQ_ERR_ARG;
  return tp_impl(kFmtNF4, x, M, K, packed_shard, absmax_shard, 0.f, bias_shard, N, rank, world,
                 y_ranks, flag_ranks, counter, epoch, static_cast<cudaStream_t>(stream), workspace,
                 workspace_bytes, y_multicast);
}

int dq_tp_linear_fp8_mc_ws(const void* x, int64_t M, int64_t K, const uint8_t* w8_shard,
                           float scale, const void* bias_shard, int64_t N, int rank, int world,
                           void* const* y_ranks, void* y_multicast,
                           unsigned int* const* flag_ranks, unsigned int* counter,
                           unsigned int epoch, void* workspace, size_t workspace_bytes,
                           dq_stream_t stream) {
  if (workspace == nullptr) return DQ_ERR_WORKSPACE;
  if (y_multicast == nullptr) return DQ_ERR_ARG;
  return tp_impl(kFmtFP8, x, M, K, w8_shard, nullptr, scale, bias_shard, N, rank, world, y_ranks,
                 flag_ranks, counter, epoch, static_cast<cudaStream_t>(stream), workspace,
                 workspace_bytes, y_multicast);
}

int dq_qk_norm_rope(const void* img, int64_t ld_img, const void* txt, int64_t ld_txt, int B,
                    int S_img, int S_txt, int H, int D, const void* w_img, const void* w_txt,
                    const float* cos_t, const float* sin_t, float eps, void* out,
                    dq_stream_t stream) {
  if (B <= 0 || S_img < 0 || S_txt < 0 || H <= 0 || D <= 0 || D % 64 != 0 || D > 256)
    return DQ_ERR_SHAPE;
  if (img == nullptr || out == nullptr || (S_txt > 0 && txt == nullptr)) return DQ_ERR_ARG;
  if ((cos_t == nullptr) != (sin_t == nullptr)) return DQ_ERR_ARG;
  // with text tokens both streams are normalized or neither
  if (S_txt > 0 && (w_img == nullptr) != (w_txt == nullptr)) return DQ_ERR_ARG;
  if (ld_img < static_cast<int64_t>(H) * D || (S_txt > 0 && ld_txt < static_cast<int64_t>(H) * D))
    return DQ_ERR_SHAPE;
  // one CTA per token, a warp per kHeadsPerWarp heads (up to 16 warps)
  const int64_t blocks = static_cast<int64_t>(B) * (S_img + S_txt);
  if (blocks == 0) return DQ_OK;
  if (blocks > INT32_MAX) return DQ_ERR_SHAPE;
  const int threads = 32 * std::min((H + kHeadsPerWarp - 1) / kHeadsPerWarp, 16);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto bf = [](const void* p) { return static_cast<const __nv_bfloat16*>(p); };
  // wide accesses when every row start is 16-byte aligned
  const bool vec = aligned(img, 16) && aligned(txt, 16) && aligned(out, 16) && aligned(w_img, 16) &&
                   aligned(w_txt, 16) && aligned(cos_t, 16) && aligned(sin_t, 16) &&
                   ld_img % 8 == 0 && (S_txt == 0 || ld_txt % 8 == 0);
  auto launch = [&](auto kern) {
    kern<<<static_cast<int>(blocks), threads, 0, st>>>(bf(img), ld_img, bf(txt), ld_txt, B, S_img, S_txt,
                                                   H, bf(w_img), bf(w_txt), cos_t, sin_t, eps,
                                                   static_cast<__nv_bfloat16*>(out));
  };
  switch (D / 32) {
    case 2: vec ? launch(qk_norm_rope_kernel<2, true>) : launch(qk_norm_rope_kernel<2, false>); break;
    case 4: vec ? launch(qk_norm_rope_kernel<4, true>) : launch(qk_norm_rope_kernel<4, false>); break;
    case 6: vec ? launch(qk_norm_rope_kernel<6, true>) : launch(qk_norm_rope_kernel<6, false>); break;
    case 8: vec ? launch(qk_norm_rope_kernel<8, true>) : launch(qk_norm_rope_kernel<8, false>); break;
    default:
      return DQ_ERR_SHAPE;
  }
  return cudaGetLastError() == cudaSuccess ? DQ_OK : DQ_ERR_LAUNCH;
}

int dq_qkv_norm_rope(int nparts, const void* const* img, const int64_t* ld_img,
                     const void* const* txt, const int64_t* ld_txt, int B, int S_img, int S_txt,
                     int H, int D, const void* const* w_img, const void* const* w_txt,
                     const int* rope, const float* cos_t, const float* sin_t, float eps,
                     void* const* out, dq_stream_t stream) {
  if (nparts < 1 || nparts > 3) return DQ_ERR_ARG;
  if (B <= 0 || S_img < 0 || S_txt < 0 || H <= 0 || D <= 0 || D % 64 != 0 || D > 256)
    return DQ_ERR_SHAPE;
  if (img == nullptr || ld_img == nullptr || out == nullptr || w_img == nullptr || w_txt == nullptr ||
      rope == nullptr || (S_txt > 0 && (txt == nullptr || ld_txt == nullptr)))
    return DQ_ERR_ARG;
  QkvParts parts = {};
  parts.nparts = nparts;
  bool vec = aligned(cos_t, 16) && aligned(sin_t, 16);
  bool any_rope = false;
  for (int p = 0; p < nparts; ++p) {
    QkvPart& P = parts.p[p];
    P.img = static_cast<const __nv_bfloat16*>(img[p]);
    P.txt = S_txt > 0 ? static_cast<const __nv_bfloat16*>(txt[p]) : nullptr;
    P.w_img = static_cast<const __nv_bfloat16*>(w_img[p]);
    P.w_txt = static_cast<const __nv_bfloat16*>(w_txt[p]);
    P.out = static_cast<__nv_bfloat16*>(out[p]);
    P.ld_img = ld_img[p];
    P.ld_txt = S_txt > 0 ? ld_txt[p] : 0;
    P.rope = rope[p] != 0;
    any_rope = any_rope || P.rope;
    if (P.img == nullptr || P.out == nullptr || (S_txt > 0 && P.txt == nullptr)) return DQ_ERR_ARG;
    // with text tokens both streams are normalized or neither
    if (S_txt > 0 && (P.w_img == nullptr) != (P.w_txt == nullptr)) return DQ_ERR_ARG;
    if (P.ld_img < static_cast<int64_t>(H) * D || (S_txt > 0 && P.ld_txt < static_cast<int64_t>(H) * D))
      return DQ_ERR_SHAPE;
    vec = vec && aligned(P.img, 16) && aligned(P.txt, 16) && aligned(P.out, 16) &&
          aligned(P.w_img, 16) && aligned(P.w_txt, 16) && P.ld_img % 8 == 0 &&
          (S_txt == 0 || P.ld_txt % 8 == 0);
  }
  if (any_rope && (cos_t == nullptr || sin_t == nullptr)) return DQ_ERR_ARG;
  const int64_t items = static_cast<int64_t>(B) * (S_img + S_txt) * nparts *
                        ((H + kHeadsPerWarp - 1) / kHeadsPerWarp);
  if (items == 0) return DQ_OK;
  DeviceInfo* d = nullptr;
  const int rc = current_device(&d);
  if (rc != DQ_OK) return rc;
  // 8 warps per CTA, at most 8 CTAs per SM: the resident grid walks the items
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((items + 7) / 8,
                                                                           static_cast<int64_t>(d->sms) * 8)));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto launch = [&](auto kern) {
    kern<<<grid, 256, 0, st>>>(parts, B, S_img, S_txt, H, cos_t, sin_t, eps);
  };
  switch (D / 32) {
    case 2: vec ? launch(qkv_norm_rope_kernel<2, true>) : launch(qkv_norm_rope_kernel<2, false>); break;
    case 4: vec ? launch(qkv_norm_rope_kernel<4, true>) : launch(qkv_norm_rope_kernel<4, false>); break;
    case 6: vec ? launch(qkv_norm_rope_kernel<6, true>) : launch(qkv_norm_rope_kernel<6, false>); break;
    case 8: vec ? launch(qkv_norm_rope_kernel<8, true>) : launch(qkv_norm_rope_kernel<8, false>); break;
    default:
      return DQ_ERR_SHAPE;
  }
  return cudaGetLastError() == cudaSuccess ? DQ_OK : DQ_ERR_LAUNCH;
}

int dq_heads_to_tokens(const void* in, int B, int H, int S_txt, int S_img, int D, void* out_txt,
                       void* out_img, dq_stream_t stream) {
  const int64_t hd = static_cast<int64_t>(H) * D;
  return dq_heads_to_tokens_ld(in, B, H, S_txt, S_img, D, out_txt, hd, out_img, hd, stream);
}

int dq_heads_to_tokens_ld(const void* in, int B, int H, int S_txt, int S_img, int D, void* out_txt,
                          int64_t ld_txt, void* out_img, int64_t ld_img, dq_stream_t stream) {
  if (B <= 0 || H <= 0 || S_txt < 0 || S_img < 0 || D <= 0 || D % 64 != 0 || D > 256)
    return DQ_ERR_SHAPE;
  if (in == nullptr || out_img == nullptr || (S_txt > 0 && out_txt == nullptr)) return DQ_ERR_ARG;
  const int64_t blocks = static_cast<int64_t>(B) * (S_img + S_txt);
  if (blocks == 0) return DQ_OK;
  if (blocks > INT32_MAX) return DQ_ERR_SHAPE;
  const int threads = 32 * std::min((H + kHeadsPerWarp - 1) / kHeadsPerWarp, 16);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const __nv_bfloat16* src = static_cast<const __nv_bfloat16*>(in);
  __nv_bfloat16* ot = static_cast<__nv_bfloat16*>(out_txt);
  __nv_bfloat16* oi = static_cast<__nv_bfloat16*>(out_img);
  if (ld_img < static_cast<int64_t>(H) * D || (S_txt > 0 && ld_txt < static_cast<int64_t>(H) * D))
    return DQ_ERR_SHAPE;
  const bool vec = aligned(in, 16) && aligned(out_txt, 16) && aligned(out_img, 16) &&
                   ld_img % 8 == 0 && (S_txt == 0 || ld_txt % 8 == 0);
  auto launch = [&](auto kern) {
    kern<<<static_cast<int>(blocks), threads, 0, st>>>(src, B, H, S_txt, S_img, ot, ld_txt, oi,
                                                       ld_img);
  };
  switch (D / 32) {
    case 2: vec ? launch(heads_to_tokens_kernel<2, true>) : launch(heads_to_tokens_kernel<2, false>); break;
    case 4: vec ? launch(heads_to_tokens_kernel<4, true>) : launch(heads_to_tokens_kernel<4, false>); break;
    case 6: vec ? launch(heads_to_tokens_kernel<6, true>) : launch(heads_to_tokens_kernel<6, false>); break;
    case 8: vec ? launch(heads_to_tokens_kernel<8, true>) : launch(heads_to_tokens_kernel<8, false>); break;
    default: return DQ_ERR_SHAPE;
  }
  return cudaGetLastError() == cudaSuccess ? DQ_OK : DQ_ERR_LAUNCH;
}

int dq_adaln_modulate(const void* x, int64_t ld_x, int64_t T, int S, int D, const void* scale,
                      const void* shift, int64_t ld_mod, float eps, void* out, int64_t ld_out,
                      dq_stream_t stream) {
  if (T < 0 || S <= 0 || D <= 0 || D % 4 != 0 || D > 8192 || T % S != 0 || T > INT32_MAX)
    return DQ_ERR_SHAPE;
  if (T == 0) return DQ_OK;
  if (x == nullptr || scale == nullptr || shift == nullptr || out == nullptr) return DQ_ERR_ARG;
  if (ld_x < D || ld_mod < D || ld_out < D || ld_x % 4 || ld_mod % 4 || ld_out % 4) return DQ_ERR_SHAPE;
  if (!aligned(x, 8) || !aligned(scale, 8) || !aligned(shift, 8) || !aligned(out, 8))
    return DQ_ERR_ALIGN;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int runs = (D / 4 + 255) / 256;  // 4-feature runs per thread
  if (runs <= 2)
    launch_adaln<2>(x, ld_x, T, S, D, scale, shift, ld_mod, eps, out, ld_out, st);
  else if (runs <= 4)
    launch_adaln<4>(x, ld_x, T, S, D, scale, shift, ld_mod, eps, out, ld_out, st);
  else
    launch_adaln<8>(x, ld_x, T, S, D, scale, shift, ld_mod, eps, out, ld_out, st);
  return cudaGetLastError() == cudaSuccess ? DQ_OK : DQ_ERR_LAUNCH;
}

int dq_gated_residual(const void* x, int64_t ld_x, const void* gate, int64_t ld_mod, const void* y,
                      int64_t ld_y, int64_t T, int S, int D, void* out, int64_t ld_out,
                      dq_stream_t stream) {
  if (T < 0 || S <= 0 || D <= 0 || D % 4 != 0 || T % S != 0) return DQ_ERR_SHAPE;
  if (T == 0) return DQ_OK;
  if (x == nullptr || gate == nullptr || y == nullptr || out == nullptr) return DQ_ERR_ARG;
  if (ld_x < D || ld_mod < D || ld_y < D || ld_out < D || ld_x % 4 || ld_mod % 4 || ld_y % 4 ||
      ld_out % 4)
    return DQ_ERR_SHAPE;
  if (!aligned(x, 8) || !aligned(gate, 8) || !aligned(y, 8) || !aligned(out, 8)) return DQ_ERR_ALIGN;
  DeviceInfo* d = nullptr;
  const int rc = current_device(&d);
  if (rc != DQ_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (D % 8 == 0 && aligned(x, 16) && aligned(gate, 16) && aligned(y, 16) && aligned(out, 16) &&
      ld_x % 8 == 0 && ld_mod % 8 == 0 && ld_y % 8 == 0 && ld_out % 8 == 0) {
    gated_residual16_kernel<<<grid_for((T * (D / 8) + 1) / 2, 256, d->sms), 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(x), ld_x, static_cast<const __nv_bfloat16*>(gate), ld_mod,
        static_cast<const __nv_bfloat16*>(y), ld_y, T, S, D, static_cast<__nv_bfloat16*>(out), ld_out);
    return cudaGetLastError() == cudaSuccess ? DQ_OK : DQ_ERR_LAUNCH;
  }
  gated_residual_kernel<<<grid_for(T * (D / 4), 256, d->sms), 256, 0, st>>>(
      static_cast<const __nv_bfloat16*>(x), ld_x, static_cast<const __nv_bfloat16*>(gate), ld_mod,
      static_cast<const __nv_bfloat16*>(y), ld_y, T, S, D, static_cast<__nv_bfloat16*>(out), ld_out);
  return cudaGetLastError() == cudaSuccess ? DQ_OK : DQ_ERR_LAUNCH;
}

int dq_device_error(int* code, dq_stream_t stream) {
  if (code == nullptr) return DQ_ERR_ARG;
  unsigned int v = 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyFromSymbolAsync(&v, g_dq_error, sizeof(v), 0, cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return DQ_ERR_CUDA;
  if (cudaStreamSynchronize(st) != cudaSuccess) return DQ_ERR_CUDA;
  const unsigned int zero = 0;
  if (v != 0 && cudaMemcpyToSymbol(g_dq_error, &zero, sizeof(zero)) != cudaSuccess) return DQ_ERR_CUDA;
  *code = (v & (1u << kErrTimeout)) ? DQ_ERR_TIMEOUT : DQ_OK;
  return DQ_OK;
}

int dq_set_pair_mode(int mode) {
  if (mode < 0 || mode > 6) return DQ_ERR_ARG;
  g_override_pair.store(mode);
  return DQ_OK;
}

int dq_set_tile_override(int bm, int splits) {
  if (bm != 0 && bm_index(bm) < 0) return DQ_ERR_ARG;
  if (splits < 0 || splits > 64) return DQ_ERR_ARG;
  g_override_bm.store(bm);
  g_override_splits.store(splits);
  return DQ_OK;
}

}  // extern "C"
