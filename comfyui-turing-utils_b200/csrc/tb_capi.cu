// C-ABI plumbing of libturing_b200: error reporting, device properties, TMA
// descriptor encoding, and the ConvRot entry points.  Argument checks mirror
// the reference binding's TORCH_CHECKs (kernel/csrc/bindings.cpp) so a caller
// sees the same conditions rejected, as a status code plus message.
#include <mutex>
#include <sstream>
#include <string>
#include <vector>

#include "tb_capi_internal.h"
#include "tb_tu.cuh"

namespace tb {

namespace {
thread_local std::string g_last_error;

std::vector<int (*)()>& error_readers() {
  static std::vector<int (*)()> readers;
  return readers;
}
std::mutex& error_readers_mutex() {
  static std::mutex m;
  return m;
}

struct DeviceInfo {
  int sm_count = 0;
  int major = 0;
  int minor = 0;
  size_t smem_optin = 0;
};

const DeviceInfo& current_device_info() {
  static std::mutex mu;
  static std::vector<DeviceInfo> infos;
  int dev = 0;
  TB_CUDA_CHECK(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  if (static_cast<int>(infos.size()) <= dev) infos.resize(dev + 1);
  DeviceInfo& d = infos[dev];
  if (d.sm_count == 0) {
    TB_CUDA_CHECK(cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev));
    TB_CUDA_CHECK(cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev));
    TB_CUDA_CHECK(cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev));
    int optin = 0;
    TB_CUDA_CHECK(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    d.smem_optin = static_cast<size_t>(optin);
  }
  return d;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      (void)cudaGetLastError();
      return nullptr;
    }
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}
}  // namespace

void set_last_error(const char* msg) { g_last_error = msg ? msg : ""; }

void throw_invalid(const char* msg) { throw Error(TB_ERR_INVALID, msg); }

void throw_cuda(cudaError_t e, const char* file, int line) {
  (void)cudaGetLastError();
  std::ostringstream s;
  s << "CUDA error: " << cudaGetErrorString(e) << " at " << file << ":" << line;
  throw Error(TB_ERR_CUDA, s.str());
}

void register_device_error_reader(int (*reader)()) {
  std::lock_guard<std::mutex> lock(error_readers_mutex());
  error_readers().push_back(reader);
}

int device_sm_count() { return current_device_info().sm_count; }
int device_cc_major() { return current_device_info().major; }
size_t device_smem_optin() { return current_device_info().smem_optin; }

void require_sm100() {
  const DeviceInfo& d = current_device_info();
  if (d.major != 10) {
    throw Error(TB_ERR_UNSUPPORTED,
                "libturing_b200 kernels are built for sm_100a (B200); the current device is not "
                "compute capability 10.x");
  }
}

void encode_tensor_map(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                       const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                       CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) throw Error(TB_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t b[5];
  cuuint32_t es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    es[i] = 1;
    if (i + 1 < rank) s[i] = strides_bytes[i];
  }
  CUresult r = fn(map, dtype, static_cast<cuuint32_t>(rank), const_cast<void*>(base), d, s, b, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    std::ostringstream m;
    m << "cuTensorMapEncodeTiled failed with CUresult " << static_cast<int>(r);
    throw Error(TB_ERR_INVALID, m.str());
  }
}

}  // namespace tb

using tb::guarded;

extern "C" {

int tb_abi_version(void) { return 1; }

const char* tb_last_error(void) { return tb::g_last_error.c_str(); }

int tb_device_error(int* code_out) {
  return guarded([&] {
    int first = 0;
    std::vector<int (*)()> readers;
    {
      std::lock_guard<std::mutex> lock(tb::error_readers_mutex());
      readers = tb::error_readers();
    }
    for (auto r : readers) {
      int v = r();
      if (v < 0) throw tb::Error(TB_ERR_CUDA, "could not read the device watchdog word");
      if (v != 0 && first == 0) first = v;
    }
    if (code_out) *code_out = first;
  });
}

// ----------------------------------------------------------- ConvRot -------

static void check_rowbuffer_args(const void* input, int64_t rows, int64_t hidden) {
  TB_REQUIRE(input != nullptr, "input must be a CUDA tensor");
  TB_REQUIRE(rows > 0 && hidden > 0 && hidden % 256 == 0,
             "BF16 row-buffer ConvRot width must be positive and divisible by 256");
  TB_REQUIRE(rows <= INT32_MAX && hidden <= INT32_MAX,
             "BF16 row-buffer ConvRot dimensions exceed the CUDA kernel range");
}

int tb_bf16_int8_convrot_quantize(const void* input, int64_t rows, int64_t hidden, int swiglu,
                                  int forced_threads, int8_t* output, float* scales,
                                  tb_stream_t stream) {
  return guarded([&] {
    TB_REQUIRE(forced_threads == 0 || forced_threads == 512 || forced_threads == 768 ||
                   forced_threads == 1024,
               "forced_threads must be 0, 512, 768, or 1024");
    check_rowbuffer_args(input, rows, hidden);
    tb::convrot_check_pointers(input, output, scales, 0, nullptr, nullptr);
    tb::require_sm100();
    tb::convrot_quantize_impl(input, TB_DTYPE_BF16, rows, hidden, swiglu ? 1 : 0, 0, 0, nullptr,
                              nullptr, output, scales, static_cast<cudaStream_t>(stream));
  });
}

int tb_bf16_int4_convrot_quantize(const void* input, int64_t rows, int64_t hidden, int swiglu,
                                  int8_t* output, float* scales, tb_stream_t stream) {
  return guarded([&] {
    check_rowbuffer_args(input, rows, hidden);
    tb::convrot_check_pointers(input, output, scales, 0, nullptr, nullptr);
    tb::require_sm100();
    tb::convrot_quantize_impl(input, TB_DTYPE_BF16, rows, hidden, swiglu ? 1 : 0, 1, 0, nullptr,
                              nullptr, output, scales, static_cast<cudaStream_t>(stream));
  });
}

int tb_bf16_gelu_int8_convrot_quantize(const void* input, int64_t rows, int64_t hidden,
                                       int8_t* output, float* scales, tb_stream_t stream) {
  return guarded([&] {
    check_rowbuffer_args(input, rows, hidden);
    tb::convrot_check_pointers(input, output, scales, 0, nullptr, nullptr);
    tb::require_sm100();
    tb::convrot_quantize_impl(input, TB_DTYPE_BF16, rows, hidden, 2, 0, 0, nullptr, nullptr,
                              output, scales, static_cast<cudaStream_t>(stream));
  });
}

int tb_bf16_gelu_int4_convrot_quantize(const void* input, int64_t rows, int64_t hidden,
                                       int8_t* output, float* scales, tb_stream_t stream) {
  return guarded([&] {
    check_rowbuffer_args(input, rows, hidden);
    tb::convrot_check_pointers(input, output, scales, 0, nullptr, nullptr);
    tb::require_sm100();
    tb::convrot_quantize_impl(input, TB_DTYPE_BF16, rows, hidden, 2, 1, 0, nullptr, nullptr,
                              output, scales, static_cast<cudaStream_t>(stream));
  });
}

static int staged_entry(const void* input, int dtype, int64_t rows, int64_t hidden, int act,
                        int int4, void* rotated, float* partial, int8_t* output, float* scales,
                        tb_stream_t stream) {
  return guarded([&] {
    TB_REQUIRE(input != nullptr, "input must be a CUDA tensor");
    TB_REQUIRE(dtype == TB_DTYPE_BF16 || dtype == TB_DTYPE_F16,
               "input must be float16 or bfloat16");
    TB_REQUIRE(rows > 0, "staged ConvRot requires at least one row");
    TB_REQUIRE(hidden > 0 && hidden % 256 == 0,
               "activated width must be positive and divisible by 256");
    TB_REQUIRE(rows <= INT32_MAX && hidden <= INT32_MAX,
               "staged ConvRot dimensions exceed the CUDA kernel range");
    TB_REQUIRE(rotated != nullptr && partial != nullptr,
               "staged ConvRot requires rotated and partial_absmax scratch");
    tb::convrot_check_pointers(input, output, scales, 1, rotated, partial);
    tb::require_sm100();
    tb::convrot_quantize_impl(input, dtype, rows, hidden, act, int4, 1, rotated, partial, output,
                              scales, static_cast<cudaStream_t>(stream));
  });
}

int tb_swiglu_int8_convrot_quantize(const void* input, int dtype, int64_t rows, int64_t hidden,
                                    void* rotated, float* partial_absmax, int8_t* output,
                                    float* scales, tb_stream_t stream) {
  return staged_entry(input, dtype, rows, hidden, 1, 0, rotated, partial_absmax, output, scales,
                      stream);
}

int tb_swiglu_int4_convrot_quantize(const void* input, int dtype, int64_t rows, int64_t hidden,
                                    void* rotated, float* partial_absmax, int8_t* output,
                                    float* scales, tb_stream_t stream) {
  return staged_entry(input, dtype, rows, hidden, 1, 1, rotated, partial_absmax, output, scales,
                      stream);
}

int tb_gelu_int8_convrot_quantize(const void* input, int dtype, int64_t rows, int64_t hidden,
                                  void* rotated, float* partial_absmax, int8_t* output,
                                  float* scales, tb_stream_t stream) {
  return staged_entry(input, dtype, rows, hidden, 2, 0, rotated, partial_absmax, output, scales,
                      stream);
}

int tb_gelu_int4_convrot_quantize(const void* input, int dtype, int64_t rows, int64_t hidden,
                                  void* rotated, float* partial_absmax, int8_t* output,
                                  float* scales, tb_stream_t stream) {
  return staged_entry(input, dtype, rows, hidden, 2, 1, rotated, partial_absmax, output, scales,
                      stream);
}

}  // extern "C"
