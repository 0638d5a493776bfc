// api_noalloc.cu -- ctts_op_linear_noalloc: the op-level linear without any
// device allocation.
//
// ctts_op_linear routes bf16 weights with >= 16 rows to the tensor cores,
// which need the activation normalized and rounded to bf16 first; it keeps
// that operand in a per-device buffer it allocates (cudaMalloc) on first use
// and grows on demand.  Callers that cannot allocate device memory -- a host
// process that owns the whole device heap through its own pool or arena, or
// a latency-critical serving loop that must not allocate once set up, where
// cudaMalloc's implicit device-wide synchronization is not acceptable -- use
// this variant instead.  Its operand lives in a file-scope __device__ array
// of fixed size, so each GPU that loads this library holds that array until
// the process exits.
//
// Like ctts_op_linear it is asynchronous on the caller's stream: a bounded
// wait inside the tensor-core kernel that gives up ends the kernel early
// (no hang) but is not reported through the return code.
#include <mutex>

#include "api_common.h"
#include "launch_state.h"

namespace {

// bf16 elements of the static operand: M * K must not exceed this (2 MiB).
constexpr size_t kNoAllocMaxElems = (size_t)1 << 20;
using ctts::kMaxDevices;

static __device__ __align__(256) uint16_t g_noalloc_operand[kNoAllocMaxElems];

// Device address of g_noalloc_operand per device.  In host code the array's
// name only stands in for the symbol; the address a kernel may use is the
// one cudaGetSymbolAddress returns with that device current.
uint16_t* g_operand_addr[kMaxDevices] = {};
std::mutex g_operand_mu;

int operand_for_current_device(uint16_t** out) {
  int dev = 0;
  CTTS_CK(cudaGetDevice(&dev));
  CTTS_REQ(dev >= 0 && dev < kMaxDevices, CTTS_ERR_RANGE, "device index out of range");
  std::lock_guard<std::mutex> lock(g_operand_mu);
  if (!g_operand_addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_operand);
    if (e != cudaSuccess || !p) {
      (void)cudaGetLastError();
      return ctts::set_error(CTTS_ERR_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    }
    g_operand_addr[dev] = static_cast<uint16_t*>(p);
  }
  *out = g_operand_addr[dev];
  return CTTS_OK;
}

}  // namespace

using namespace ctts;

extern "C" int ctts_op_linear_noalloc(const float* x, int M, int K, const void* w, int w_dtype, int N,
                                      const float* norm_w, float eps, const float* res, float* y,
                                      void* stream) {
  CTTS_REQ(x && w && y && M >= 0 && K > 0 && N > 0, CTTS_ERR_ARG, "bad argument");
  CTTS_REQ(w_dtype == CTTS_F32 || w_dtype == CTTS_BF16, CTTS_ERR_ARG, "bad weight dtype");
  CTTS_REQ(K % (w_dtype == CTTS_BF16 ? 8 : 4) == 0, CTTS_ERR_ARG, "K must be a multiple of 4 (f32) / 8 (bf16)");
  cudaStream_t s = as_stream(stream, 0);
  if (w_dtype == CTTS_BF16 && M >= 16 && K % 64 == 0) {
    CTTS_REQ((size_t)M * K <= kNoAllocMaxElems, CTTS_ERR_RANGE,
             "M*K = " + std::to_string((size_t)M * K) + " exceeds the static operand of " +
                 std::to_string(kNoAllocMaxElems) + " bf16 elements");
    uint16_t* xb = nullptr;
    int rc = operand_for_current_device(&xb);
    if (rc) return rc;
    PrepArgs pa;
    pa.x = x; pa.x_ld = K; pa.y = xb; pa.y_ld = K; pa.M = M; pa.K = K; pa.norm_w = norm_w; pa.eps = eps;
    CTTS_CK(launch_prep_bf16(pa, s));
    TcArgs e;
    e.y = y;
    e.y_ld = N;
    e.res = res;
    TcScratch none;  // the split-K partials live in the cluster's shared memory
    return tc_run(none, xb, M, K, w, N, e, s, nullptr);
  }
  // CUDA-core path: no operand copy, nothing to hold
  LinearArgs a;
  a.x = x; a.x_ld = K; a.M = M; a.K = K; a.N = N; a.w = w; a.w_bf16 = w_dtype == CTTS_BF16;
  a.y = y; a.y_ld = N; a.norm_w = norm_w; a.eps = eps; a.res = res;
  CTTS_CK(launch_linear(a, s));
  return CTTS_OK;
}
