// Split-K ternary GEMV of libivonar_b200.so: a variant of ivb_ternary_gemv for long inputs that
// spreads the input columns over more CTAs. Each CTA writes the partial row sums of its column block
// to a static device scratch (one slot per column block and row, so nothing is accumulated in place),
// and the epilogue adds a row's partials in column-block order: the result does not depend on which
// CTA finishes first. The entry point allocates nothing: the scratch is a file-scope __device__ array
// whose address is looked up once per device (cudaGetSymbolAddress).
#include <cuda_runtime.h>

#include <mutex>

#include "ivb_common.h"
#include "ivb_device.cuh"

size_t ivb_gemv_smem_bytes(int n);

namespace ivb {

constexpr int kSplitMaxRows = 32768;    // rows of the scratch
constexpr int kSplitMaxIn = 16384;      // input length (each CTA quantises it in shared memory)
constexpr int kSplitChunks = 16;        // 64-input chunks per CTA column block (1024 inputs)
constexpr int kSplitRows = 64;          // rows per CTA row block
constexpr int kSplitMaxBlocks = (kSplitMaxIn / 64 + kSplitChunks - 1) / kSplitChunks;  // column blocks (16)

// partial row sums [column block][row] (2 MB of fp32), and [0]: the activation scale of the call
static __device__ __align__(256) float g_split_part[kSplitMaxBlocks * kSplitMaxRows];
static __device__ __align__(256) float g_split_scale[4];

// Grid (row blocks, column blocks). Every CTA quantises the whole input (the scale needs the
// whole vector; same canonical quantiser as ivb_ternary_gemv), then writes, for each of its rows,
// the sum over its chunks of (integer chunk dot) * group scale to g_split_part[column block][row].
__global__ void __launch_bounds__(kThreads) splitk_partial_kernel(const IvbTernary m, const float* x, const float* norm_w,
                                                                  float norm_eps, float clip, float act_eps) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int n = m.in_features;
  const int pad = ((n + 63) >> 6) << 6;
  float* xv = reinterpret_cast<float*>(smem);
  int8_t* act = reinterpret_cast<int8_t*>(xv + pad);
  int* xs = reinterpret_cast<int*>(act + pad);
  float* red = reinterpret_cast<float*>(xs + (pad >> 6));
  load_vector(x, n, xv);
  __syncthreads();
  const float s = quantize_block(xv, n, norm_w, norm_eps, clip, act_eps, act, true, xs, red);
  if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) g_split_scale[0] = s;
  const int chunks = pad >> 6;
  const int u0 = blockIdx.y * kSplitChunks, u1 = min(chunks, u0 + kSplitChunks);
  const int r0 = blockIdx.x * kSplitRows, r1 = min(m.rows, r0 + kSplitRows);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // a half-warp per row: lanes 0-15 and 16-31 take rows rb and rb + 1, one chunk per lane (the loop
  // bound is uniform across the warp, so every lane reaches the shuffles)
  const int half = lane >> 4, hl = lane & 15;
  for (int rb = r0 + 2 * warp; rb < r1; rb += 2 * kWarps) {
    const int r = rb + half;
    float part = 0.0f;
    const int u = u0 + hl;
    if (r < r1 && u < u1) {
      const uint4 w = __ldg(reinterpret_cast<const uint4*>(m.packed + static_cast<size_t>(r) * m.row_bytes) + u);
      const float sc = h2f(__ldg(m.scales + static_cast<size_t>(r) * m.scale_stride + (u >> 1)));
      part = static_cast<float>(chunk_dot(w, act, u) - xs[u]) * sc;
    }
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) part += __shfl_xor_sync(kFull, part, off);
    if (hl == 0 && r < r1) g_split_part[static_cast<size_t>(blockIdx.y) * kSplitMaxRows + r] = part;
  }
}

// out[r] from the partial sums (added in column-block order): act_scale, bias and the epilogue of
// ivb_ternary_gemv.
__global__ void __launch_bounds__(kThreads) splitk_epilogue_kernel(const float* bias, int rows, int blocks, int epilogue,
                                                                   float* out) {
  const int i = blockIdx.x * kThreads + threadIdx.x;
  const float s = g_split_scale[0];
  auto value = [&](int r) {
    float acc = g_split_part[r];
    for (int b = 1; b < blocks; ++b) acc += g_split_part[static_cast<size_t>(b) * kSplitMaxRows + r];
    float v = acc * s;
    if (bias != nullptr) v += __ldg(bias + r);
    return v;
  };
  if (epilogue == IVB_EPI_SILU_PAIR) {
    if (2 * i + 1 < rows) out[i] = silu_f(value(2 * i)) * value(2 * i + 1);
  } else if (i < rows) {
    out[i] = epilogue == IVB_EPI_RESIDUAL ? out[i] + value(i) : value(i);
  }
}

struct SplitDevice {
  float* part = nullptr;
  bool ready = false;
};

// Once per device, with that device current: the scratch address (the first call also loads the
// module there) and the partial kernel's shared-memory limit for the longest input it accepts.
static int32_t split_device(int dev, float** part) {
  static std::mutex lock;
  static SplitDevice table[64];
  if (dev < 0 || dev >= 64) return fail(IVB_EINVAL, "ivb_ternary_gemv_splitk: device %d out of range", dev);
  std::lock_guard<std::mutex> guard(lock);
  if (!table[dev].ready) {
    void* p = nullptr;
    IVB_CUDA(cudaGetSymbolAddress(&p, g_split_part));
    IVB_CUDA(cudaFuncSetAttribute(splitk_partial_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(ivb_gemv_smem_bytes(kSplitMaxIn))));
    table[dev].part = static_cast<float*>(p);
    table[dev].ready = true;
  }
  *part = table[dev].part;
  return IVB_OK;
}

}  // namespace ivb

extern "C" {

int32_t ivb_ternary_gemv_splitk(const IvbTernary* m, const float* x, const float* norm_weight, float norm_eps,
                                float norm_clip, float act_eps, int32_t epilogue, float* out, void* stream) {
  using namespace ivb;
  if (m == nullptr || x == nullptr || out == nullptr) return fail(IVB_EINVAL, "ivb_ternary_gemv_splitk: null argument");
  if (int32_t rc = check_ternary(*m, "ivb_ternary_gemv_splitk")) return rc;
  if (epilogue < IVB_EPI_STORE || epilogue > IVB_EPI_SILU_PAIR)
    return fail(IVB_EINVAL, "ivb_ternary_gemv_splitk: bad epilogue");
  if (epilogue == IVB_EPI_SILU_PAIR && (m->rows & 1))
    return fail(IVB_EINVAL, "ivb_ternary_gemv_splitk: silu pairs need an even row count");
  if (m->rows > kSplitMaxRows)
    return fail(IVB_EINVAL, "ivb_ternary_gemv_splitk: %d rows exceed the %d-row static scratch", m->rows, kSplitMaxRows);
  if (m->in_features > kSplitMaxIn)
    return fail(IVB_EINVAL, "ivb_ternary_gemv_splitk: %d inputs exceed the %d-input limit", m->in_features, kSplitMaxIn);
  int dev = 0;
  IVB_CUDA(cudaGetDevice(&dev));
  float* part = nullptr;
  if (int32_t rc = split_device(dev, &part)) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t smem = ivb_gemv_smem_bytes(m->in_features);
  const int chunks = (m->in_features + 63) / 64;
  const int blocks = (chunks + kSplitChunks - 1) / kSplitChunks;
  const dim3 grid((m->rows + kSplitRows - 1) / kSplitRows, blocks);
  splitk_partial_kernel<<<grid, kThreads, smem, s>>>(*m, x, norm_weight, norm_eps, norm_clip, act_eps);
  IVB_CUDA(cudaGetLastError());
  const int outs = epilogue == IVB_EPI_SILU_PAIR ? m->rows / 2 : m->rows;
  splitk_epilogue_kernel<<<(outs + kThreads - 1) / kThreads, kThreads, 0, s>>>(m->bias, m->rows, blocks, epilogue, out);
  IVB_CUDA(cudaGetLastError());
  return IVB_OK;
}

}  // extern "C"
