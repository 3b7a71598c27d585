// Unit entry points of libivonar_b200.so: activation quantiser, exact integer group dots,
// fused norm + quantise + ternary GEMV, sampler, and the bounded-wait probe.
// Each is one kernel launch built from the device blocks in ivb_device.cuh, the same code the
// persistent decoder runs.
#include <cuda_runtime.h>

#include <cstring>
#include <string>

#include "ivb_common.h"
#include "ivb_device.cuh"

namespace ivb {

namespace {
thread_local std::string g_last_error;
}

int32_t fail(int32_t code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error.assign(buf);
  return code;
}

int32_t check_ternary(const IvbTernary& m, const char* name) {
  if (m.packed == nullptr || m.scales == nullptr) return fail(IVB_EINVAL, "%s: null packed or scales pointer", name);
  if (m.rows <= 0 || m.in_features <= 0) return fail(IVB_EINVAL, "%s: empty matrix (%d x %d)", name, m.rows, m.in_features);
  const int need_bytes = (m.in_features + 3) / 4;
  if (m.row_bytes < need_bytes || (m.row_bytes & 15) != 0)
    return fail(IVB_EINVAL, "%s: row_bytes %d must be >= %d and a multiple of 16", name, m.row_bytes, need_bytes);
  const int chunks = (m.in_features + 63) / 64;
  if (m.row_bytes < chunks * 16)
    return fail(IVB_EINVAL, "%s: row_bytes %d must cover %d 16-byte chunks", name, m.row_bytes, chunks);
  const int groups = (m.in_features + 127) / 128;
  if (m.scale_stride < groups) return fail(IVB_EINVAL, "%s: scale_stride %d < %d groups", name, m.scale_stride, groups);
  if ((reinterpret_cast<uintptr_t>(m.packed) & 15) != 0) return fail(IVB_EINVAL, "%s: packed pointer not 16-byte aligned", name);
  return IVB_OK;
}

bool device_is_sm100() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return false;
  if (cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) return false;
  return major == 10 && minor == 0;
}

// ------------------------------------------------------------------------------------------------
// kernels
// ------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) quantize_kernel(const float* x, const float* norm_w, int n, float norm_eps,
                                                            float clip, float act_eps, int8_t* q8, float* scale,
                                                            int32_t* xsum) {
  extern __shared__ __align__(16) unsigned char smem[];
  float* xv = reinterpret_cast<float*>(smem);
  const int pad = ((n + 63) >> 6) << 6;
  int* xs = reinterpret_cast<int*>(xv + pad);
  float* red = reinterpret_cast<float*>(xs + (pad >> 6));
  int8_t* codes = reinterpret_cast<int8_t*>(red + 64);
  for (int i = threadIdx.x; i < n; i += kThreads) xv[i] = x[i];
  __syncthreads();
  const float s = quantize_block(xv, n, norm_w, norm_eps, clip, act_eps, codes, false, xs, red);
  for (int i = threadIdx.x; i < n; i += kThreads) q8[i] = codes[i];
  if (xsum != nullptr)
    for (int u = threadIdx.x; u < (pad >> 6); u += kThreads) xsum[u] = xs[u];
  if (threadIdx.x == 0) *scale = s;
}

// One thread per (row, group): the integer core of the GEMV, through the production chunk_dot.
__global__ void __launch_bounds__(kThreads) group_dots_kernel(const IvbTernary m, const int8_t* q8, int32_t* dots,
                                                              int groups) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int n = m.in_features;
  const int chunks = (n + 63) >> 6;
  int8_t* act = reinterpret_cast<int8_t*>(smem);
  int* xs = reinterpret_cast<int*>(smem + (chunks << 6));
  for (int i = threadIdx.x; i < (chunks << 6); i += kThreads) act[act_slot(i)] = i < n ? q8[i] : 0;
  __syncthreads();
  for (int u = threadIdx.x; u < chunks; u += kThreads) {
    const int* words = reinterpret_cast<const int*>(act + (u << 6));
    int total = 0;
    for (int w = 0; w < 16; ++w) total = __dp4a(words[w], 0x01010101, total);
    xs[u] = total;
  }
  __syncthreads();
  const long long item = static_cast<long long>(blockIdx.x) * kThreads + threadIdx.x;
  if (item >= static_cast<long long>(m.rows) * groups) return;
  const int row = static_cast<int>(item / groups), g = static_cast<int>(item % groups);
  const uint4* wrow = reinterpret_cast<const uint4*>(m.packed + static_cast<size_t>(row) * m.row_bytes);
  int total = 0;
  for (int u = 2 * g; u < min(2 * g + 2, chunks); ++u) total += chunk_dot(__ldg(wrow + u), act, u) - xs[u];
  dots[item] = total;
}

struct GemvSmem {
  static size_t bytes(int n) {
    const size_t pad = static_cast<size_t>((n + 63) / 64) * 64;
    return pad * 4 + pad + (pad / 64) * 4 + 64 * 4 + 2 * kThreads * 4 + 16;
  }
};

// One CTA per row block; each CTA (norm +) quantises the input itself, then runs gemv_rows.
__global__ void __launch_bounds__(kThreads, 1) gemv_kernel(const IvbTernary m, const float* x, const float* norm_w,
                                                           float norm_eps, float clip, float act_eps, int epilogue,
                                                           float* out, int rows_per_cta, int lpr_log) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int n = m.in_features;
  const int pad = ((n + 63) >> 6) << 6;
  float* xv = reinterpret_cast<float*>(smem);
  int8_t* act = reinterpret_cast<int8_t*>(xv + pad);
  int* xs = reinterpret_cast<int*>(act + pad);
  float* red = reinterpret_cast<float*>(xs + (pad >> 6));
  float* res = red + 64;
  const GemvGeom g = gemv_geom(m, rows_per_cta, lpr_log, blockIdx.x);
  uint4 pf[kPrefetch];
  float pfs[kPrefetch];
  gemv_prefetch(m, g, pf, pfs);
  load_vector(x, n, xv);
  __syncthreads();
  const float s = quantize_block(xv, n, norm_w, norm_eps, clip, act_eps, act, true, xs, red);
  gemv_rows(m, g, act, xs, s, epilogue, out, pf, pfs, res, nullptr);
}

__global__ void __launch_bounds__(kThreads, 1) sample_kernel(const float* logits, uint8_t* seen, int vocab,
                                                             const float* sampling, const int64_t* top_k, int max_top_k,
                                                             uint64_t* rng, int64_t* token, int64_t* history) {
  extern __shared__ __align__(16) unsigned char smem[];
  SampleSmem sm;
  carve_sample(smem, vocab, sm);
  sample_block(logits, seen, vocab, sampling, top_k, max_top_k, rng, token, history, sm);
}

__global__ void probe_wait_kernel(unsigned* counter, unsigned* error_word, unsigned long long timeout_ns) {
  __shared__ int flag;
  Sync s{counter, error_word, timeout_ns};
  // Arrive once and wait for a second arrival that nobody makes: the bounded wait must give up.
  grid_barrier(s, 2u, &flag);
}


// ---- checkpoint ingest: validation of the packed buffers on the device ---------------------------
// Grid (blocks, buffers). Packed ternary bytes: a 2-bit field holding the reserved code 3 has both of its
// bits set, so (b & (b >> 1) & 0x55) != 0 finds it (loader.py:94-112); fp16 scales must be finite
// (exponent field not all ones) and positive (sign clear, not zero). The lowest offending buffer index
// per test goes to bad[0] (code 3), bad[1] (not finite), bad[2] (not positive) by atomicMin.
// bad[0..2] = count: "no buffer failed" for each of the three checks.
__global__ void validate_init_kernel(int32_t* bad, int32_t count) {
  if (threadIdx.x < 3) bad[threadIdx.x] = count;
}

__global__ void validate_buffers_kernel(const IvbCheckBuffer* bufs, int32_t* bad) {
  const IvbCheckBuffer b = bufs[blockIdx.y];
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const long long i0 = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  bool code3 = false, nonfinite = false, nonpositive = false;
  if (b.kind == IVB_CHECK_PACKED) {
    const unsigned char* q = static_cast<const unsigned char*>(b.data);
    const long long n16 = (reinterpret_cast<uintptr_t>(q) & 15) == 0 ? b.count / 16 : 0;
    const uint4* q4 = reinterpret_cast<const uint4*>(q);
    for (long long i = i0; i < n16; i += stride) {
      const uint4 v = __ldg(q4 + i);
      const unsigned m = (v.x & (v.x >> 1)) | (v.y & (v.y >> 1)) | (v.z & (v.z >> 1)) | (v.w & (v.w >> 1));
      code3 |= (m & 0x55555555u) != 0u;
    }
    for (long long i = 16 * n16 + i0; i < b.count; i += stride) {
      const unsigned v = __ldg(q + i);
      code3 |= (v & (v >> 1) & 0x55u) != 0u;
    }
  } else {
    const unsigned short* h = static_cast<const unsigned short*>(b.data);
    for (long long i = i0; i < b.count; i += stride) {
      const unsigned v = __ldg(h + i);
      nonfinite |= (v & 0x7C00u) == 0x7C00u;
      nonpositive |= (v & 0x8000u) != 0u || (v & 0x7FFFu) == 0u;
    }
  }
  if (__syncthreads_or(code3) && threadIdx.x == 0) atomicMin(bad, static_cast<int32_t>(blockIdx.y));
  if (__syncthreads_or(nonfinite) && threadIdx.x == 0) atomicMin(bad + 1, static_cast<int32_t>(blockIdx.y));
  if (__syncthreads_or(nonpositive) && threadIdx.x == 0) atomicMin(bad + 2, static_cast<int32_t>(blockIdx.y));
}

}  // namespace ivb

size_t ivb_sample_smem_bytes(int vocab) { return ivb::sample_smem_bytes(vocab); }

size_t ivb_gemv_smem_bytes(int n) { return ivb::GemvSmem::bytes(n); }

int ivb_lpr_log(int in_features) {
  const int chunks = (in_features + 63) / 64;
  int lg = 0;
  while ((1 << lg) < chunks && lg < 5) ++lg;
  return lg;
}

// ------------------------------------------------------------------------------------------------
// C ABI
// ------------------------------------------------------------------------------------------------
extern "C" {

int32_t ivb_abi_version(void) { return IVB_ABI_VERSION; }

const char* ivb_last_error(void) { return ivb::g_last_error.c_str(); }

int32_t ivb_device_supported(void) { return ivb::device_is_sm100() ? 1 : 0; }

int32_t ivb_quantize(const float* x, const float* norm_weight, int32_t n, float norm_eps, float norm_clip,
                     float act_eps, int8_t* q8, float* scale, int32_t* xsum, void* stream) {
  using namespace ivb;
  if (x == nullptr || q8 == nullptr || scale == nullptr || n <= 0) return fail(IVB_EINVAL, "ivb_quantize: bad arguments");
  const size_t pad = align_up(n, 64);
  const size_t smem = pad * 4 + (pad / 64) * 4 + 64 * 4 + pad + 16;
  if (smem > 200 * 1024) return fail(IVB_EINVAL, "ivb_quantize: n = %d is too large", n);
  IVB_CUDA(cudaFuncSetAttribute(quantize_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  quantize_kernel<<<1, kThreads, smem, static_cast<cudaStream_t>(stream)>>>(x, norm_weight, n, norm_eps, norm_clip,
                                                                             act_eps, q8, scale, xsum);
  IVB_CUDA(cudaGetLastError());
  return IVB_OK;
}

int32_t ivb_ternary_group_dots(const IvbTernary* m, const int8_t* q8, int32_t* dots, void* stream) {
  using namespace ivb;
  if (m == nullptr || q8 == nullptr || dots == nullptr) return fail(IVB_EINVAL, "ivb_ternary_group_dots: null argument");
  if (int32_t rc = check_ternary(*m, "ivb_ternary_group_dots")) return rc;
  const int groups = (m->in_features + 127) / 128;
  const size_t chunks = (m->in_features + 63) / 64;
  const size_t smem = chunks * 64 + chunks * 4 + 16;
  if (smem > 200 * 1024) return fail(IVB_EINVAL, "ivb_ternary_group_dots: in_features too large");
  IVB_CUDA(cudaFuncSetAttribute(group_dots_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  const long long items = static_cast<long long>(m->rows) * groups;
  const int grid = static_cast<int>((items + kThreads - 1) / kThreads);
  group_dots_kernel<<<grid, kThreads, smem, static_cast<cudaStream_t>(stream)>>>(*m, q8, dots, groups);
  IVB_CUDA(cudaGetLastError());
  return IVB_OK;
}

int32_t ivb_ternary_gemv(const IvbTernary* m, const float* x, const float* norm_weight, float norm_eps,
                         float norm_clip, float act_eps, int32_t epilogue, float* out, void* stream) {
  using namespace ivb;
  if (m == nullptr || x == nullptr || out == nullptr) return fail(IVB_EINVAL, "ivb_ternary_gemv: null argument");
  if (int32_t rc = check_ternary(*m, "ivb_ternary_gemv")) return rc;
  if (epilogue < IVB_EPI_STORE || epilogue > IVB_EPI_SILU_PAIR) return fail(IVB_EINVAL, "ivb_ternary_gemv: bad epilogue");
  if (epilogue == IVB_EPI_SILU_PAIR && (m->rows & 1)) return fail(IVB_EINVAL, "ivb_ternary_gemv: silu pairs need an even row count");
  const size_t smem = GemvSmem::bytes(m->in_features);
  if (smem > 200 * 1024) return fail(IVB_EINVAL, "ivb_ternary_gemv: in_features too large");
  int dev = 0, sms = 148;
  IVB_CUDA(cudaGetDevice(&dev));
  IVB_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int lpr_log = ivb_lpr_log(m->in_features);
  int per = (m->rows + sms - 1) / sms;
  if (per & 1) ++per;
  const int grid = (m->rows + per - 1) / per;
  IVB_CUDA(cudaFuncSetAttribute(gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  gemv_kernel<<<grid, kThreads, smem, static_cast<cudaStream_t>(stream)>>>(*m, x, norm_weight, norm_eps, norm_clip,
                                                                           act_eps, epilogue, out, per, lpr_log);
  IVB_CUDA(cudaGetLastError());
  return IVB_OK;
}

int32_t ivb_sample(const float* logits, uint8_t* seen, int32_t vocab, const float* sampling, const int64_t* top_k,
                   int32_t max_top_k, uint64_t* rng, int64_t* token, int64_t* history, void* stream) {
  using namespace ivb;
  if (logits == nullptr || seen == nullptr || sampling == nullptr || top_k == nullptr || rng == nullptr || token == nullptr)
    return fail(IVB_EINVAL, "ivb_sample: null argument");
  if (vocab <= 0 || max_top_k <= 0) return fail(IVB_EINVAL, "ivb_sample: bad vocab or max_top_k");
  const size_t smem = ivb_sample_smem_bytes(vocab);
  if (smem > 227 * 1024) return fail(IVB_EINVAL, "ivb_sample: vocab %d does not fit the on-chip sampler", vocab);
  IVB_CUDA(cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  sample_kernel<<<1, kThreads, smem, static_cast<cudaStream_t>(stream)>>>(logits, seen, vocab, sampling, top_k,
                                                                          max_top_k, rng, token, history);
  IVB_CUDA(cudaGetLastError());
  return IVB_OK;
}

int32_t ivb_probe_wait_timeout(uint32_t* counter, uint32_t* error_word, uint64_t timeout_ns, void* stream) {
  using namespace ivb;
  if (counter == nullptr || error_word == nullptr) return fail(IVB_EINVAL, "ivb_probe_wait_timeout: null argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  IVB_CUDA(cudaMemsetAsync(counter, 0, sizeof(uint32_t), s));
  IVB_CUDA(cudaMemsetAsync(error_word, 0, sizeof(uint32_t), s));
  probe_wait_kernel<<<1, 32, 0, s>>>(counter, error_word, timeout_ns == 0 ? 1000000000ull : timeout_ns);
  IVB_CUDA(cudaGetLastError());
  IVB_CUDA(cudaStreamSynchronize(s));
  uint32_t word = 0;
  IVB_CUDA(cudaMemcpy(&word, error_word, sizeof(word), cudaMemcpyDeviceToHost));
  if (word != 0) return fail(static_cast<int32_t>(word), "bounded wait gave up (device error word %u)", word);
  return IVB_OK;
}

int32_t ivb_validate_buffers(const IvbCheckBuffer* buffers, int32_t count, int32_t* bad, void* stream) {
  using namespace ivb;
  if (buffers == nullptr || bad == nullptr || count <= 0 || count > 65535) return fail(IVB_EINVAL, "ivb_validate_buffers: bad argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  validate_init_kernel<<<1, 32, 0, s>>>(bad, count);
  IVB_CUDA(cudaGetLastError());
  validate_buffers_kernel<<<dim3(64, count), 256, 0, s>>>(buffers, bad);
  IVB_CUDA(cudaGetLastError());
  return IVB_OK;
}

}  // extern "C"
