// C-ABI layer and host runtime of libfelix_b200.so: per-device state, tensor-map
// encoding, library-owned scratch, error reporting, the device watchdog word,
// and the extern "C" entry points declared in include/felix_c.h.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <utility>

#include "felix_internal.h"
#include "sm100_ptx.cuh"

// Watchdog word, one per device (each device holds its own copy of a __device__
// variable). Its device address is looked up once per device.
__device__ unsigned g_felix_watchdog_word;

namespace felix_impl {

namespace {
thread_local int t_last_cuda = 0;
thread_local std::string t_last_msg;

std::mutex g_mu;
DeviceInfo g_dev[64];
bool g_dev_ready[64] = {false};

struct WsEntry {
  void* ptr = nullptr;
  size_t bytes = 0;
};
std::map<std::pair<int, cudaStream_t>, WsEntry> g_ws;

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;
std::once_flag g_encode_once;

void load_encode() {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
          cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_encode = reinterpret_cast<EncodeTiledFn>(fn);
}
}  // namespace

FelixCode api_error(const char* msg, cudaError_t e) {
  t_last_cuda = int(e);
  t_last_msg = msg ? msg : "";
  return FelixCode{FELIX_API_ERROR, e};
}

FelixCode launch_error(cudaError_t e, const char* msg) {
  t_last_cuda = int(e);
  t_last_msg = std::string(msg ? msg : "") + ": " + cudaGetErrorString(e);
  return FelixCode{FELIX_KERNEL_LAUNCH_FAILED, e};
}

DeviceInfo* current_device_info() {
  int d = -1;
  if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_dev_ready[d]) {
    DeviceInfo& di = g_dev[d];
    di.ordinal = d;
    if (cudaDeviceGetAttribute(&di.num_sms, cudaDevAttrMultiProcessorCount, d) != cudaSuccess)
      return nullptr;
    cudaDeviceGetAttribute(&di.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, d);
    void* addr = nullptr;
    if (cudaGetSymbolAddress(&addr, g_felix_watchdog_word) != cudaSuccess) return nullptr;
    di.status_word = static_cast<unsigned*>(addr);
    g_dev_ready[d] = true;
  }
  return &g_dev[d];
}

void* library_workspace(DeviceInfo* dev, cudaStream_t stream, size_t bytes) {
  std::lock_guard<std::mutex> lk(g_mu);
  WsEntry& w = g_ws[{dev->ordinal, stream}];
  if (w.bytes >= bytes) return w.ptr;
  if (w.ptr) {
    // The old buffer may still be in use by work queued on this stream.
    cudaStreamSynchronize(stream);
    cudaFree(w.ptr);
    w.ptr = nullptr;
    w.bytes = 0;
  }
  size_t sz = bytes < (size_t(1) << 20) ? (size_t(1) << 20) : bytes;
  if (cudaMalloc(&w.ptr, sz) != cudaSuccess) {
    w.ptr = nullptr;
    return nullptr;
  }
  if (cudaMemsetAsync(w.ptr, 0, sz, stream) != cudaSuccess) return nullptr;
  w.bytes = sz;
  return w.ptr;
}

static int encode_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                     uint64_t pitch, uint32_t bi, uint32_t bo, CUtensorMapSwizzle sw) {
  std::call_once(g_encode_once, load_encode);
  if (!g_encode) return -1;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {pitch};
  cuuint32_t box[2] = {bi, bo};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : int(r);
}

int encode_tmap_2d_f16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                       uint64_t pitch, uint32_t bi, uint32_t bo) {
  return encode_2d(map, base, inner, outer, pitch, bi, bo, CU_TENSOR_MAP_SWIZZLE_128B);
}
int encode_tmap_2d_f16_swizzle(CUtensorMap* map, const void* base, uint64_t inner,
                               uint64_t outer, uint64_t pitch, uint32_t bi, uint32_t bo,
                               int swizzle_bytes) {
  CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_NONE;
  if (swizzle_bytes == 32) sw = CU_TENSOR_MAP_SWIZZLE_32B;
  else if (swizzle_bytes == 64) sw = CU_TENSOR_MAP_SWIZZLE_64B;
  else if (swizzle_bytes == 128) sw = CU_TENSOR_MAP_SWIZZLE_128B;
  return encode_2d(map, base, inner, outer, pitch, bi, bo, sw);
}

int encode_tmap_3d_f16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer1,
                       uint64_t outer2, uint64_t pitch1, uint64_t pitch2, uint32_t bi,
                       uint32_t bo1, uint32_t bo2) {
  std::call_once(g_encode_once, load_encode);
  if (!g_encode) return -1;
  cuuint64_t dims[3] = {inner, outer1, outer2};
  cuuint64_t strides[2] = {pitch1, pitch2};
  cuuint32_t box[3] = {bi, bo1, bo2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : int(r);
}

int encode_tmap_3d_f32(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer1,
                       uint64_t outer2, uint64_t pitch1, uint64_t pitch2, uint32_t bi,
                       uint32_t bo1, uint32_t bo2) {
  std::call_once(g_encode_once, load_encode);
  if (!g_encode) return -1;
  cuuint64_t dims[3] = {inner, outer1, outer2};
  cuuint64_t strides[2] = {pitch1, pitch2};
  cuuint32_t box[3] = {bi, bo1, bo2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : int(r);
}

int encode_tmap_2d_f32(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                       uint64_t pitch, uint32_t bi, uint32_t bo, bool swizzle128) {
  std::call_once(g_encode_once, load_encode);
  if (!g_encode) return -1;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {pitch};
  cuuint32_t box[2] = {bi, bo};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : int(r);
}

int encode_tmap_2d_f16_noswizzle(CUtensorMap* map, const void* base, uint64_t inner,
                                 uint64_t outer, uint64_t pitch, uint32_t bi, uint32_t bo) {
  return encode_2d(map, base, inner, outer, pitch, bi, bo, CU_TENSOR_MAP_SWIZZLE_NONE);
}

__global__ void scale_half_kernel(__half* c, size_t n, float beta) {
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n;
       i += size_t(gridDim.x) * blockDim.x)
    c[i] = beta == 0.f ? __float2half_rn(0.f) : __float2half_rn(beta * __half2float(c[i]));
}
__global__ void scale_float_kernel(float* c, size_t n, float beta) {
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n;
       i += size_t(gridDim.x) * blockDim.x)
    c[i] = beta == 0.f ? 0.f : beta * c[i];
}

FelixCode scale_half_matrix(__half* C, size_t n, float beta, cudaStream_t stream) {
  if (n == 0) return FelixCode{FELIX_SUCCESS, cudaSuccess};
  scale_half_kernel<<<592, 256, 0, stream>>>(C, n, beta);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return launch_error(e, "scale");
  return FelixCode{FELIX_SUCCESS, cudaSuccess};
}
FelixCode scale_float_matrix(float* C, size_t n, float beta, cudaStream_t stream) {
  if (n == 0) return FelixCode{FELIX_SUCCESS, cudaSuccess};
  scale_float_kernel<<<592, 256, 0, stream>>>(C, n, beta);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return launch_error(e, "scale");
  return FelixCode{FELIX_SUCCESS, cudaSuccess};
}

// One CTA waits on an mbarrier that nothing arrives on; the bounded wait gives
// up after limit_ns, records kWdProbe in the watchdog word and the kernel
// returns. Exercises the same wait routine the GEMM/attention kernels use.
__global__ void watchdog_probe_kernel(unsigned* status, unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    felix_sm100::mbar_init(&bar, 1);
    abort_flag = 0;
    felix_sm100::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0)
    felix_sm100::mbar_wait(&bar, 0, &abort_flag, status, felix_sm100::kWdProbe, limit_ns);
  __syncthreads();
}

FelixCode watchdog_probe_launch(uint32_t limit_us, cudaStream_t stream) {
  if (limit_us == 0 || limit_us > 1000000) return api_error("watchdog_probe: limit_us in 1..1e6");
  DeviceInfo* dev = current_device_info();
  if (!dev) return launch_error(cudaGetLastError(), "watchdog_probe: no device");
  watchdog_probe_kernel<<<1, 32, 0, stream>>>(dev->status_word,
                                              (unsigned long long)limit_us * 1000ull);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return launch_error(e, "watchdog_probe");
  return FelixCode{FELIX_SUCCESS, cudaSuccess};
}

static int finish(FelixCode c) {
  if (c.type == FELIX_SUCCESS) {
    t_last_cuda = 0;
    t_last_msg.clear();
  }
  return c.type;
}

}  // namespace felix_impl

using namespace felix_impl;

extern "C" {

int felix_last_cuda_error(void) { return t_last_cuda; }
const char* felix_last_error_message(void) { return t_last_msg.c_str(); }
const char* felix_version(void) { return "sion-b200 0.1 (sm_100a)"; }

int felix_num_sms(int* count) {
  DeviceInfo* d = current_device_info();
  if (!d) return launch_error(cudaGetLastError(), "no device").type;
  if (count) *count = d->num_sms;
  return FELIX_SUCCESS;
}

int felix_sgemm(uint32_t M, uint32_t N, uint32_t K, float alpha, const float* A, const float* B,
                float beta, float* C, void* stream) {
  SgemmOptions o;
  return finish(sgemm_launch(M, N, K, alpha, A, B, beta, C, o, nullptr, 0,
                             static_cast<cudaStream_t>(stream)));
}

int felix_sgemm_ex(uint32_t M, uint32_t N, uint32_t K, float alpha, const float* A,
                   const float* B, float beta, float* C, int split_k, void* workspace,
                   size_t workspace_bytes, void* stream) {
  if (split_k < 0) return api_error("sgemm: split_k must be >= 0").type;
  SgemmOptions o;
  o.split_k = split_k;
  return finish(sgemm_launch(M, N, K, alpha, A, B, beta, C, o, workspace, workspace_bytes,
                             static_cast<cudaStream_t>(stream)));
}

int felix_sgemm_noalloc(uint32_t M, uint32_t N, uint32_t K, float alpha, const float* A,
                        const float* B, float beta, float* C, int split_k, void* stream) {
  return finish(sgemm_noalloc_launch(M, N, K, alpha, A, B, beta, C, split_k,
                                     static_cast<cudaStream_t>(stream)));
}

int felix_sgemm_workspace_size(uint32_t M, uint32_t N, uint32_t K, int split_k, size_t* bytes) {
  DeviceInfo* d = current_device_info();
  if (!d) return launch_error(cudaGetLastError(), "no device").type;
  SgemmOptions o;
  o.split_k = split_k;
  if (bytes) *bytes = sgemm_workspace_bytes(M, N, K, o, d->num_sms);
  return FELIX_SUCCESS;
}

int felix_hgemm(uint32_t M, uint32_t N, uint32_t K, float alpha, const void* A, const void* B,
                float beta, void* C, int b_layout, void* stream) {
  if (b_layout != FELIX_B_KN && b_layout != FELIX_B_NK)
    return api_error("hgemm: b_layout must be FELIX_B_KN or FELIX_B_NK").type;
  HgemmOptions o;
  return finish(hgemm_launch(M, N, K, alpha, static_cast<const __half*>(A),
                             static_cast<const __half*>(B), beta, static_cast<__half*>(C),
                             b_layout == FELIX_B_KN, o, nullptr, 0,
                             static_cast<cudaStream_t>(stream)));
}

int felix_hgemm_ex(uint32_t M, uint32_t N, uint32_t K, float alpha, const void* A, const void* B,
                   float beta, void* C, int b_layout, int block_n, int stream_k, int max_ctas,
                   void* workspace, size_t workspace_bytes, void* stream) {
  if (b_layout != FELIX_B_KN && b_layout != FELIX_B_NK)
    return api_error("hgemm: b_layout must be FELIX_B_KN or FELIX_B_NK").type;
  if (stream_k < 0 || stream_k > 2) return api_error("hgemm: stream_k must be 0, 1 or 2").type;
  if (max_ctas < 0) return api_error("hgemm: max_ctas must be >= 0").type;
  HgemmOptions o;
  o.block_n = block_n;
  o.stream_k = stream_k;
  o.max_ctas = max_ctas;
  return finish(hgemm_launch(M, N, K, alpha, static_cast<const __half*>(A),
                             static_cast<const __half*>(B), beta, static_cast<__half*>(C),
                             b_layout == FELIX_B_KN, o, workspace, workspace_bytes,
                             static_cast<cudaStream_t>(stream)));
}

int felix_hgemm_ex2(uint32_t M, uint32_t N, uint32_t K, float alpha, const void* A, const void* B,
                    float beta, void* C, int b_layout, int block_n, int stream_k, int max_ctas,
                    int cta_pair, void* workspace, size_t workspace_bytes, void* stream) {
  if (b_layout != FELIX_B_KN && b_layout != FELIX_B_NK)
    return api_error("hgemm: b_layout must be FELIX_B_KN or FELIX_B_NK").type;
  if (stream_k < 0 || stream_k > 2) return api_error("hgemm: stream_k must be 0, 1 or 2").type;
  if (max_ctas < 0) return api_error("hgemm: max_ctas must be >= 0").type;
  if (cta_pair < 0 || cta_pair > 2) return api_error("hgemm: cta_pair must be 0, 1 or 2").type;
  if (cta_pair == 2 && block_n != 0 && block_n != 256)
    return api_error("hgemm: CTA pairs use 256-wide tiles (block_n 0 or 256)").type;
  HgemmOptions o;
  o.block_n = block_n;
  o.stream_k = stream_k;
  o.max_ctas = max_ctas;
  o.cta_pair = cta_pair;
  return finish(hgemm_launch(M, N, K, alpha, static_cast<const __half*>(A),
                             static_cast<const __half*>(B), beta, static_cast<__half*>(C),
                             b_layout == FELIX_B_KN, o, workspace, workspace_bytes,
                             static_cast<cudaStream_t>(stream)));
}

int felix_hgemm_workspace_size2(uint32_t M, uint32_t N, uint32_t K, int block_n, int stream_k,
                                int max_ctas, int cta_pair, size_t* bytes) {
  DeviceInfo* d = current_device_info();
  if (!d) return launch_error(cudaGetLastError(), "no device").type;
  HgemmOptions o;
  o.block_n = block_n;
  o.stream_k = stream_k;
  o.max_ctas = max_ctas;
  o.cta_pair = cta_pair;
  if (bytes) *bytes = hgemm_workspace_bytes(M, N, K, o, d->num_sms);
  return FELIX_SUCCESS;
}

int felix_hgemm_workspace_size(uint32_t M, uint32_t N, uint32_t K, int block_n, int stream_k,
                               int max_ctas, size_t* bytes) {
  DeviceInfo* d = current_device_info();
  if (!d) return launch_error(cudaGetLastError(), "no device").type;
  HgemmOptions o;
  o.block_n = block_n;
  o.stream_k = stream_k;
  o.max_ctas = max_ctas;
  if (bytes) *bytes = hgemm_workspace_bytes(M, N, K, o, d->num_sms);
  return FELIX_SUCCESS;
}

int felix_flash_attn_fwd(const void* Q, const void* K, const void* V, void* O, float* lse,
                         uint32_t heads, uint32_t batch, uint32_t seqlen, uint32_t head_dim,
                         float scale, void* stream) {
  return finish(flash_attn_launch(static_cast<const __half*>(Q), static_cast<const __half*>(K),
                                  static_cast<const __half*>(V), static_cast<__half*>(O), lse,
                                  heads, batch, seqlen, head_dim, scale, false,
                                  static_cast<cudaStream_t>(stream)));
}

int felix_flash_attn_fwd_ex(const void* Q, const void* K, const void* V, void* O, float* lse,
                            uint32_t heads, uint32_t batch, uint32_t seqlen, uint32_t head_dim,
                            float scale, int causal, void* stream) {
  return finish(flash_attn_launch(static_cast<const __half*>(Q), static_cast<const __half*>(K),
                                  static_cast<const __half*>(V), static_cast<__half*>(O), lse,
                                  heads, batch, seqlen, head_dim, scale, causal != 0,
                                  static_cast<cudaStream_t>(stream)));
}

int felix_flash_attn_bwd(const void* Q, const void* K, const void* V, const void* O,
                         const void* dO, const float* lse, void* dQ, void* dK, void* dV,
                         uint32_t heads, uint32_t batch, uint32_t seqlen, uint32_t head_dim,
                         float scale, int causal, void* workspace, size_t workspace_bytes,
                         void* stream) {
  return finish(flash_attn_bwd_launch(
      static_cast<const __half*>(Q), static_cast<const __half*>(K), static_cast<const __half*>(V),
      static_cast<const __half*>(O), static_cast<const __half*>(dO), lse,
      static_cast<__half*>(dQ), static_cast<__half*>(dK), static_cast<__half*>(dV), heads, batch,
      seqlen, head_dim, scale, causal != 0, workspace, workspace_bytes,
      static_cast<cudaStream_t>(stream)));
}

int felix_flash_attn_bwd_workspace_size(uint32_t heads, uint32_t batch, uint32_t seqlen,
                                        uint32_t head_dim, size_t* bytes) {
  if (bytes) *bytes = flash_attn_bwd_workspace_bytes(heads, batch, seqlen, head_dim);
  return FELIX_SUCCESS;
}

int felix_topk_select(const float* data, float* out, uint32_t num_slices, uint32_t slice_size,
                      uint32_t k, int largest, void* stream) {
  return finish(topk_select_launch(data, out, num_slices, slice_size, k, largest != 0,
                                   static_cast<cudaStream_t>(stream)));
}

int felix_watchdog_status(unsigned* code, int clear) {
  DeviceInfo* d = current_device_info();
  if (!d) return launch_error(cudaGetLastError(), "no device").type;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return launch_error(e, "watchdog_status: device sync").type;
  unsigned v = 0;
  e = cudaMemcpy(&v, d->status_word, sizeof(v), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return launch_error(e, "watchdog_status: read").type;
  if (clear) {
    unsigned z = 0;
    e = cudaMemcpy(d->status_word, &z, sizeof(z), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return launch_error(e, "watchdog_status: clear").type;
  }
  if (code) *code = v;
  if (v != 0) {
    t_last_cuda = 0;
    t_last_msg = "device watchdog: a bounded wait gave up (site " + std::to_string(v) + ")";
    return FELIX_KERNEL_RUNTIME_ERROR;
  }
  return finish(FelixCode{FELIX_SUCCESS, cudaSuccess});
}

int felix_watchdog_probe(uint32_t limit_us, void* stream) {
  return finish(watchdog_probe_launch(limit_us, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
