// Exact-erf GELU (optionally bias-fused) and SwiGLU for sm_100a.
//
// Reference semantics (VideoLingo-user native/asr/src):
//   gelu (engine.cu:110-112)          0.5f*x*(1+erff(x*0.70710678118654752440f))
//   gelu_kernel (engine.cu:194-198)   x = half(gelu(float(x))), in place
//   add_bias_kernel (engine.cu:200-205) x = half(float(x) + float(b[col]))
//   silu_mul_kernel (decoder.cu:103-109) g = half(g / (1 + __expf(-g)) * u)
// Both are pure streams: 16-byte vector loads, several vectors in flight per
// thread, grid sized to a whole number of waves over the SMs.
//
// GELU for 16-bit storage types runs as a table lookup: an input is one of
// 65536 bit patterns, so the library builds, once per device, a 128 KB table
// per type holding round(gelu(x)) for every pattern - computed on the device
// with the very expression above, so the result is bit-identical to
// evaluating erff per element - and each block stages the table in shared
// memory.  That replaces ~29 instructions per element (erff plus conversions
// saturate the special-function pipe) by ~3, leaving the kernel HBM-bound.
#include <mutex>
#include <type_traits>

#include "vl_common.cuh"
#include "vl_kernels.h"

namespace vl {
namespace {

constexpr int kActThreads = 256;
constexpr int kUnroll = 4;  // 16-byte vectors in flight per thread

__device__ __forceinline__ float gelu_erf(float x) {
  return 0.5f * x * (1.0f + erff(x * 0.70710678118654752440f));
}

// The reference divides with IEEE `/`; __fdividef (reciprocal + multiply,
// within 2 ulp of it in fp32) halves the instruction count of this
// issue-bound stream.  For g < -88 both give 0 after rounding to the storage
// type (the true value is below 1e-36).
__device__ __forceinline__ float silu_mul(float g, float u) {
  return __fdividef(g, 1.0f + __expf(-g)) * u;
}

// Contiguous GELU without bias: flat grid-stride over 16-byte vectors.
template <typename T>
__global__ void __launch_bounds__(kActThreads)
    gelu_flat_kernel(const T* in, T* out, int64_t nvec) {
  using S = Storage<T>;
  constexpr int E = S::kVec;
  const uint4* src = reinterpret_cast<const uint4*>(in);
  uint4* dst = reinterpret_cast<uint4*>(out);
  const int64_t step = static_cast<int64_t>(gridDim.x) * kActThreads * kUnroll;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * kActThreads * kUnroll + threadIdx.x;
       base < nvec; base += step) {
    uint4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = base + u * kActThreads;
      if (i < nvec) v[u] = ld_stream(src + i);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = base + u * kActThreads;
      if (i < nvec) {
        float f[E];
        S::unpack(v[u], f);
#pragma unroll
        for (int e = 0; e < E; ++e) f[e] = gelu_erf(f[e]);
        st_stream(dst + i, S::pack(f));
      }
    }
  }
}

// Row-structured GELU with bias: blockIdx.y strides rows, threads cover the
// row's vectors.  t = round(x + b) is formed before GELU, as the reference
// stores the biased activation before gelu_kernel reads it.
template <typename T>
__global__ void __launch_bounds__(kActThreads)
    gelu_bias_kernel(const T* in, const T* __restrict__ bias, T* out, int64_t rows,
                     int vec_per_row) {
  using S = Storage<T>;
  constexpr int E = S::kVec;
  const int v = blockIdx.x * kActThreads + threadIdx.x;
  if (v >= vec_per_row) return;
  float b[E];
  S::unpack(__ldg(reinterpret_cast<const uint4*>(bias) + v), b);
  for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) {
    const int64_t i = r * vec_per_row + v;
    float f[E];
    S::unpack(ld_stream(reinterpret_cast<const uint4*>(in) + i), f);
#pragma unroll
    for (int e = 0; e < E; ++e) f[e] = gelu_erf(S::round_trip(f[e] + b[e]));
    st_stream(reinterpret_cast<uint4*>(out) + i, S::pack(f));
  }
}

// Any shape / alignment.
template <typename T>
__global__ void gelu_scalar_kernel(const T* in, const T* bias, T* out, int64_t rows,
                                   int64_t cols) {
  using S = Storage<T>;
  const int64_t n = rows * cols;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float x = S::to_float(in[i]);
    if (bias) x = S::round_trip(x + S::to_float(bias[i % cols]));
    out[i] = S::from_float(gelu_erf(x));
  }
}

template <typename T>
__global__ void __launch_bounds__(kActThreads)
    swiglu_flat_kernel(const T* gate, const T* up, T* out, int64_t nvec) {
  using S = Storage<T>;
  constexpr int E = S::kVec;
  const uint4* g4 = reinterpret_cast<const uint4*>(gate);
  const uint4* u4 = reinterpret_cast<const uint4*>(up);
  uint4* o4 = reinterpret_cast<uint4*>(out);
  const int64_t step = static_cast<int64_t>(gridDim.x) * kActThreads * kUnroll;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * kActThreads * kUnroll + threadIdx.x;
       base < nvec; base += step) {
    uint4 gv[kUnroll], uv[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = base + u * kActThreads;
      if (i < nvec) {
        gv[u] = ld_stream(g4 + i);
        uv[u] = ld_stream(u4 + i);
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = base + u * kActThreads;
      if (i < nvec) {
        float g[E], x[E];
        S::unpack(gv[u], g);
        S::unpack(uv[u], x);
#pragma unroll
        for (int e = 0; e < E; ++e) g[e] = silu_mul(g[e], x[e]);
        st_stream(o4 + i, S::pack(g));
      }
    }
  }
}

// Strided rows (packed gate|up layouts): blockIdx.y strides rows.
template <typename T>
__global__ void __launch_bounds__(kActThreads)
    swiglu_rows_kernel(const T* gate, const T* up, T* out, int64_t rows, int vec_per_row,
                       int64_t gs, int64_t us, int64_t os) {
  using S = Storage<T>;
  constexpr int E = S::kVec;
  const int v = blockIdx.x * kActThreads + threadIdx.x;
  if (v >= vec_per_row) return;
  for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) {
    float g[E], x[E];
    S::unpack(ld_stream(reinterpret_cast<const uint4*>(gate + r * gs) + v), g);
    S::unpack(ld_stream(reinterpret_cast<const uint4*>(up + r * us) + v), x);
#pragma unroll
    for (int e = 0; e < E; ++e) g[e] = silu_mul(g[e], x[e]);
    st_stream(reinterpret_cast<uint4*>(out + r * os) + v, S::pack(g));
  }
}

template <typename T>
__global__ void swiglu_scalar_kernel(const T* gate, const T* up, T* out, int64_t rows,
                                     int64_t cols, int64_t gs, int64_t us, int64_t os) {
  using S = Storage<T>;
  const int64_t n = rows * cols;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / cols, c = i % cols;
    out[r * os + c] = S::from_float(silu_mul(S::to_float(gate[r * gs + c]),
                                             S::to_float(up[r * us + c])));
  }
}

// ---------------------------------------------------------------------------
// Table GELU (bf16 / fp16)
// ---------------------------------------------------------------------------
// One block per SM (the table fills 128 KB of smem).  512 threads x 8
// vectors in flight measured best among {1024, 768, 512} threads x
// {4, 6, 8} vectors, with and without software pipelining: fewer warps
// contending for the table's banks beat more warps (94 % of the measured HBM
// copy bandwidth at 7.86 GB per launch, 5 % above 1024 x 8).
constexpr int kLutThreads = 512;
constexpr int kLutUnroll = 8;              // 16-byte vectors in flight per thread (64 KB per SM)
constexpr int kLutEntries = 65536;
constexpr int kLutBytes = kLutEntries * 2;
constexpr int64_t kLutMinElems = 1 << 20;  // below this the table load does not pay off

// [0]: bf16 bits -> bf16 bits of round(gelu(x)); [1]: the same for fp16.
static __device__ __align__(16) uint16_t g_gelu_lut[2][kLutEntries];

template <typename T>
struct LutSlot;
template <>
struct LutSlot<__nv_bfloat16> {
  static constexpr int kIndex = 0;
};
template <>
struct LutSlot<__half> {
  static constexpr int kIndex = 1;
};

__global__ void gelu_lut_init_kernel(uint16_t* lut) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= kLutEntries) return;
  // Same conversion and packing instructions as the direct kernels.
  const float xb = bf16_lo(static_cast<uint32_t>(i));
  lut[i] = static_cast<uint16_t>(pack_bf16x2(gelu_erf(xb), 0.f) & 0xffffu);
  const float xh = __half2float(__ushort_as_half(static_cast<unsigned short>(i)));
  lut[kLutEntries + i] = static_cast<uint16_t>(pack_f16x2(gelu_erf(xh), 0.f) & 0xffffu);
}

template <typename T, bool kBias>
__global__ void __launch_bounds__(kLutThreads, 1)
    gelu_lut_kernel(const T* in, const T* __restrict__ bias, T* out, int64_t nvec,
                    uint32_t vec_per_row, const uint16_t* __restrict__ lut_global) {
  using S = Storage<T>;
  constexpr int E = S::kVec;
  extern __shared__ __align__(16) unsigned char lut_raw[];
  {
    uint4* dst = reinterpret_cast<uint4*>(lut_raw);
    const uint4* src = reinterpret_cast<const uint4*>(lut_global);
#pragma unroll 4
    for (int i = threadIdx.x; i < kLutBytes / 16; i += kLutThreads) dst[i] = __ldg(src + i);
  }
  __syncthreads();
  const uint16_t* lut = reinterpret_cast<const uint16_t*>(lut_raw);
  const uint4* src = reinterpret_cast<const uint4*>(in);
  uint4* dst = reinterpret_cast<uint4*>(out);
  const uint4* bvec = reinterpret_cast<const uint4*>(bias);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kLutThreads;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * kLutThreads + threadIdx.x; base < nvec;
       base += stride * kLutUnroll) {
    uint4 v[kLutUnroll];
#pragma unroll
    for (int u = 0; u < kLutUnroll; ++u) {
      const int64_t i = base + u * stride;
      if (i < nvec) v[u] = ld_stream(src + i);
    }
#pragma unroll
    for (int u = 0; u < kLutUnroll; ++u) {
      const int64_t i = base + u * stride;
      if (i < nvec) {
        uint4 w = v[u];
        if (kBias) {
          float x[E], b[E];
          S::unpack(w, x);
          S::unpack(__ldg(bvec + static_cast<uint32_t>(i) % vec_per_row), b);
#pragma unroll
          for (int e = 0; e < E; ++e) x[e] = x[e] + b[e];
          w = S::pack(x);  // round(x + b), as the reference stores it before GELU
        }
        uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t lo = lut[words[j] & 0xffffu];
          const uint32_t hi = lut[words[j] >> 16];
          words[j] = lo | (hi << 16);
        }
        st_stream(dst + i, make_uint4(words[0], words[1], words[2], words[3]));
      }
    }
  }
}

struct LutState {
  std::mutex mu;
  int state = 0;  // 0 = not built, 1 = ready, 2 = unavailable
  uint16_t* ptr = nullptr;
};
LutState g_lut_state[64];

// Device address of the GELU tables on the current device, building them on
// first use: a private stream runs the init kernel and is synchronised once,
// so every later launch on any stream sees a complete table.  Returns null -
// and the caller evaluates erff directly, with identical results - while the
// caller's stream is being captured before the table exists, or if building
// it failed.
const uint16_t* gelu_table(cudaStream_t stream) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  LutState& st = g_lut_state[dev];
  std::lock_guard<std::mutex> lock(st.mu);
  if (st.state == 1) return st.ptr;
  if (st.state == 2) return nullptr;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) {
    (void)cudaGetLastError();
    return nullptr;
  }
  void* p = nullptr;
  cudaStream_t s = nullptr;
  cudaError_t err = cudaGetSymbolAddress(&p, g_gelu_lut);
  if (err == cudaSuccess)
    err = cudaFuncSetAttribute(gelu_lut_kernel<__nv_bfloat16, false>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, kLutBytes);
  if (err == cudaSuccess)
    err = cudaFuncSetAttribute(gelu_lut_kernel<__nv_bfloat16, true>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, kLutBytes);
  if (err == cudaSuccess)
    err = cudaFuncSetAttribute(gelu_lut_kernel<__half, false>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, kLutBytes);
  if (err == cudaSuccess)
    err = cudaFuncSetAttribute(gelu_lut_kernel<__half, true>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, kLutBytes);
  if (err == cudaSuccess) err = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
  if (err == cudaSuccess) {
    gelu_lut_init_kernel<<<kLutEntries / 256, 256, 0, s>>>(static_cast<uint16_t*>(p));
    err = cudaGetLastError();
    if (err == cudaSuccess) err = cudaStreamSynchronize(s);
  }
  if (s != nullptr) cudaStreamDestroy(s);
  if (err != cudaSuccess) {
    (void)cudaGetLastError();
    st.state = 2;
    return nullptr;
  }
  st.ptr = static_cast<uint16_t*>(p);
  st.state = 1;
  return st.ptr;
}

template <typename T>
bool gelu_via_table(const void* in, const void* bias, void* out, int64_t rows, int64_t cols,
                    cudaStream_t stream) {
  constexpr int E = Storage<T>::kVec;
  const int64_t n = rows * cols;
  if (n < kLutMinElems || n % E != 0 || !aligned16(in) || !aligned16(out)) return false;
  if (bias != nullptr && (!aligned16(bias) || cols % E != 0 || n / E >= (int64_t(1) << 32)))
    return false;
  const uint16_t* table = gelu_table(stream);
  if (table == nullptr) return false;
  table += LutSlot<T>::kIndex * kLutEntries;
  const int64_t nvec = n / E;
  int64_t blocks =
      (nvec + int64_t(kLutThreads) * kLutUnroll - 1) / (int64_t(kLutThreads) * kLutUnroll);
  if (blocks > sm_count()) blocks = sm_count();
  const uint32_t vpr = bias ? static_cast<uint32_t>(cols / E) : 1u;
  if (bias)
    gelu_lut_kernel<T, true><<<static_cast<unsigned>(blocks), kLutThreads, kLutBytes, stream>>>(
        static_cast<const T*>(in), static_cast<const T*>(bias), static_cast<T*>(out), nvec, vpr,
        table);
  else
    gelu_lut_kernel<T, false><<<static_cast<unsigned>(blocks), kLutThreads, kLutBytes, stream>>>(
        static_cast<const T*>(in), nullptr, static_cast<T*>(out), nvec, vpr, table);
  return true;
}

// Grid of a grid-stride stream kernel: enough blocks for the data, at most
// the number resident at once (a single persistent wave, no tail wave).
unsigned flat_blocks(const void* kernel, int64_t nvec) {
  const int64_t per_block = static_cast<int64_t>(kActThreads) * kUnroll;
  const int64_t need = (nvec + per_block - 1) / per_block;
  const int64_t cap = resident_blocks(kernel, kActThreads, 0);
  return static_cast<unsigned>(need < cap ? (need > 0 ? need : 1) : cap);
}

dim3 row_grid(int vec_per_row, int64_t rows) {
  const unsigned gx = static_cast<unsigned>((vec_per_row + kActThreads - 1) / kActThreads);
  const int64_t want = (static_cast<int64_t>(sm_count()) * 8 + gx - 1) / gx;
  int64_t gy = rows < want ? rows : want;
  if (gy > 65535) gy = 65535;
  if (gy < 1) gy = 1;
  return dim3(gx, static_cast<unsigned>(gy), 1);
}

template <typename T>
cudaError_t gelu_typed(const void* in, const void* bias, void* out, int64_t rows, int64_t cols,
                       cudaStream_t stream) {
  constexpr int E = Storage<T>::kVec;
  const T* x = static_cast<const T*>(in);
  T* y = static_cast<T*>(out);
  if constexpr (!std::is_same<T, float>::value) {
    if (gelu_via_table<T>(in, bias, out, rows, cols, stream)) return cudaGetLastError();
  }
  const bool vec_ok = aligned16(in) && aligned16(out) && (bias == nullptr || aligned16(bias));
  if (bias == nullptr && vec_ok && ((rows * cols) % E == 0)) {
    const int64_t nvec = rows * cols / E;
    gelu_flat_kernel<T><<<flat_blocks(reinterpret_cast<const void*>(gelu_flat_kernel<T>), nvec),
                           kActThreads, 0, stream>>>(x, y, nvec);
  } else if (bias != nullptr && vec_ok && cols % E == 0 && cols / E < (1 << 30)) {
    const int vpr = static_cast<int>(cols / E);
    gelu_bias_kernel<T><<<row_grid(vpr, rows), kActThreads, 0, stream>>>(
        x, static_cast<const T*>(bias), y, rows, vpr);
  } else {
    const int64_t n = rows * cols;
    int64_t blocks = (n + kActThreads - 1) / kActThreads;
    const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
    if (blocks > cap) blocks = cap;
    gelu_scalar_kernel<T><<<static_cast<unsigned>(blocks), kActThreads, 0, stream>>>(
        x, static_cast<const T*>(bias), y, rows, cols);
  }
  return cudaGetLastError();
}

template <typename T>
cudaError_t swiglu_typed(const void* gate, const void* up, void* out, int64_t rows, int64_t cols,
                         int64_t gs, int64_t us, int64_t os, cudaStream_t stream) {
  constexpr int E = Storage<T>::kVec;
  const T* g = static_cast<const T*>(gate);
  const T* u = static_cast<const T*>(up);
  T* o = static_cast<T*>(out);
  const bool vec_ok = aligned16(gate) && aligned16(up) && aligned16(out) && cols % E == 0 &&
                      gs % E == 0 && us % E == 0 && os % E == 0;
  if (vec_ok && gs == cols && us == cols && os == cols) {
    const int64_t nvec = rows * cols / E;
    swiglu_flat_kernel<T><<<flat_blocks(reinterpret_cast<const void*>(swiglu_flat_kernel<T>), nvec),
                             kActThreads, 0, stream>>>(g, u, o, nvec);
  } else if (vec_ok && cols / E < (1 << 30)) {
    const int vpr = static_cast<int>(cols / E);
    swiglu_rows_kernel<T><<<row_grid(vpr, rows), kActThreads, 0, stream>>>(g, u, o, rows, vpr, gs,
                                                                          us, os);
  } else {
    const int64_t n = rows * cols;
    int64_t blocks = (n + kActThreads - 1) / kActThreads;
    const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
    if (blocks > cap) blocks = cap;
    swiglu_scalar_kernel<T><<<static_cast<unsigned>(blocks), kActThreads, 0, stream>>>(
        g, u, o, rows, cols, gs, us, os);
  }
  return cudaGetLastError();
}

}  // namespace

cudaError_t prepare_gelu() {
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  cudaError_t err = cudaStreamIsCapturing(nullptr, &cap);
  if (err != cudaSuccess) return err;
  if (cap != cudaStreamCaptureStatusNone) return cudaErrorStreamCaptureUnsupported;
  return gelu_table(nullptr) != nullptr ? cudaSuccess : cudaErrorUnknown;
}

cudaError_t launch_gelu(const void* in, const void* bias, void* out, int64_t rows, int64_t cols,
                        int dtype, cudaStream_t stream) {
  if (rows == 0 || cols == 0) return cudaSuccess;
  switch (dtype) {
    case kDtypeF32: return gelu_typed<float>(in, bias, out, rows, cols, stream);
    case kDtypeF16: return gelu_typed<__half>(in, bias, out, rows, cols, stream);
    default: return gelu_typed<__nv_bfloat16>(in, bias, out, rows, cols, stream);
  }
}

cudaError_t launch_swiglu(const void* gate, const void* up, void* out, int64_t rows, int64_t cols,
                          int64_t gate_stride, int64_t up_stride, int64_t out_stride, int dtype,
                          cudaStream_t stream) {
  if (rows == 0 || cols == 0) return cudaSuccess;
  switch (dtype) {
    case kDtypeF32:
      return swiglu_typed<float>(gate, up, out, rows, cols, gate_stride, up_stride, out_stride, stream);
    case kDtypeF16:
      return swiglu_typed<__half>(gate, up, out, rows, cols, gate_stride, up_stride, out_stride, stream);
    default:
      return swiglu_typed<__nv_bfloat16>(gate, up, out, rows, cols, gate_stride, up_stride,
                                         out_stride, stream);
  }
}

}  // namespace vl
