// Host-side helpers shared by the translation units of libivonar_b200.so.
#pragma once

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <utility>

#include "ivonar_b200.h"

namespace ivb {

// Records the message returned by ivb_last_error() on this thread; returns `code`.
int32_t fail(int32_t code, const char* fmt, ...);

// Maps a CUDA error to IVB_ECUDA with the call site in the message.
inline int32_t cuda_fail(cudaError_t err, const char* what) {
  return fail(IVB_ECUDA, "%s: %s (%s)", what, cudaGetErrorString(err), cudaGetErrorName(err));
}

#define IVB_CUDA(call)                                     \
  do {                                                     \
    cudaError_t ivb_err_ = (call);                         \
    if (ivb_err_ != cudaSuccess) return ivb::cuda_fail(ivb_err_, #call); \
  } while (0)

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Programmatic dependent launch: the grid may be scheduled while the previous kernel on the stream is
// still running (once that kernel's CTAs have all triggered, or exited). The kernel must run
// pdl_enter() (or griddepcontrol.wait) before it reads anything an earlier kernel wrote.
template <typename... Params, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Checks the layout contract of one ternary matrix (row_bytes 16-aligned and wide enough,
// scale_stride covers ceil(in/128) groups, 16-byte aligned base pointer).
int32_t check_ternary(const IvbTernary& m, const char* name);

// True when the current device is compute capability 10.0 (B200 / sm_100a).
bool device_is_sm100();

// ivb_ternary_gemm with the split-K partial sums in `partial` (partial_floats floats of device memory;
// nullptr: no split): ivb_decoder_prefill and ivb_batch_decode pass a slice of their own workspace, so
// their calls share nothing with other calls on the device.
constexpr size_t kGemmPartialFloats = size_t(1) << 22;
int32_t ternary_gemm_into(const IvbTernary* m, const int8_t* q8, int32_t ldq, const float* act_scale, int32_t rows_t,
                          int32_t epilogue, float* out, int32_t ldo, uint32_t* error, float* partial, size_t partial_floats,
                          void* stream);

// The model description a decoder handle was created from (layers: its host array), and the device
// error word that ivb_decoder_check reports.
const IvbModelDesc& decoder_model(const IvbDecoder* dec, const IvbLayerDesc** layers);
unsigned* decoder_error_word(const IvbDecoder* dec);

}  // namespace ivb
