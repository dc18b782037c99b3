// Allocation-free MatMulNBits prefill (b2m_matmul_nbits_noalloc).
//
// Some callers cannot call cudaMalloc at the point where they run an operator:
// a host application that has handed all device memory to its own pool up
// front (and accounts every byte against it), or an inference loop that must
// never risk an out-of-memory failure or the device-wide synchronisation that
// cudaMalloc / cudaFree can cause in the middle of a run. For them this entry
// point runs the same tcgen05 prefill kernels as b2m_matmul_nbits with FAST
// numerics, but its only working memory is the file-scope array below:
// static device memory that is reserved when the library's module is loaded
// onto a device and held by that device until the process exits. The caller
// supplies A, bias and Y and the prepacked weight; nothing is allocated.
#include <mutex>

#include "b2m_internal.cuh"

namespace {

// Working memory of b2m_matmul_nbits_noalloc: the f16 copy of the activations
// (M x roundup(K, 8) halves) followed by the device error word of the kernel's
// bounded waits.
constexpr size_t kErrOffset = B2M_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_noalloc_scratch[B2M_NOALLOC_SCRATCH_BYTES + 256];

// Device address of g_noalloc_scratch, resolved once per device. In host code
// the array's name is only a host-side stand-in for the symbol, so it must
// never be passed to a kernel directly.
constexpr int kMaxDevices = 64;
std::mutex g_mu;
void *g_addr[kMaxDevices] = {nullptr};

void *scratch_address(int device) {
  B2M_REQUIRE(device >= 0 && device < kMaxDevices, B2M_ERR_NO_DEVICE, "device ordinal out of range");
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_addr[device]) {
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      (void)cudaGetLastError();
      b2m_throw(B2M_ERR_CUDA, std::string("b2m_matmul_nbits_noalloc: cudaGetSymbolAddress failed: ") +
                                  cudaGetErrorString(e));
    }
    g_addr[device] = p;
  }
  return g_addr[device];
}

}  // namespace

extern "C" B2M_API b2m_status b2m_matmul_nbits_noalloc(const b2m_weight *w, const float *a, int64_t m,
                                                       const float *bias, float *y, void *stream) {
  try {
    B2M_REQUIRE(w && w->kind == W_NBITS, B2M_ERR_INVALID_ARGUMENT,
                "MatMulNBits no-alloc: weight is not a MatMulNBits weight");
    B2M_REQUIRE(m >= 0 && (a || m == 0) && (y || m == 0), B2M_ERR_INVALID_ARGUMENT,
                "MatMulNBits no-alloc: bad pointers");
    if (m == 0) return B2M_OK;
    const int64_t need = m * nbits_tc_k8(w->k) * 2;
    if (need > (int64_t)B2M_NOALLOC_SCRATCH_BYTES)
      b2m_throw(B2M_ERR_INVALID_ARGUMENT,
                "MatMulNBits no-alloc: M x roundup(K, 8) x 2 = " + std::to_string(need) +
                    " bytes of activations exceed the fixed " + std::to_string((long long)B2M_NOALLOC_SCRATCH_BYTES) +
                    "-byte scratch; split M into smaller calls");
    B2M_REQUIRE(nbits_tc_supported(w->nb, m, w->k, w->n), B2M_ERR_UNSUPPORTED,
                "MatMulNBits no-alloc: shape not supported by the tensor-core kernel");
    int prev = -1;
    B2M_CUDA(cudaGetDevice(&prev));
    const int dev = w->ctx->device;
    if (prev != dev) B2M_CUDA(cudaSetDevice(dev));
    struct Restore {
      int p, d;
      ~Restore() {
        if (p >= 0 && p != d) cudaSetDevice(p);
      }
    } restore{prev, dev};
    unsigned char *base = static_cast<unsigned char *>(scratch_address(dev));
    int32_t *err = reinterpret_cast<int32_t *>(base + kErrOffset);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // The error word must start at zero; the activation region is fully
    // rewritten by the conversion kernel, so it needs no clearing.
    B2M_CUDA(cudaMemsetAsync(err, 0, sizeof(int32_t), s));
    NbitsArgs p;
    p.A = a;
    p.w = &w->nb;
    p.bias = bias;
    p.Y = y;
    p.M = m;
    p.K = w->k;
    p.N = w->n;
    p.dev_err = err;
    launch_nbits_tc(p, reinterpret_cast<__half *>(base), s);
    int32_t host_err = 0;
    B2M_CUDA(cudaMemcpyAsync(&host_err, err, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
    B2M_CUDA(cudaStreamSynchronize(s));
    if (host_err != B2M_DEVERR_NONE)
      b2m_throw(B2M_ERR_TIMEOUT, "MatMulNBits no-alloc: a bounded device-side wait timed out");
    return B2M_OK;
  } catch (const B2mError &e) {
    b2m_set_last_error(e.msg);
    return e.code;
  } catch (...) {
    b2m_set_last_error("MatMulNBits no-alloc: unexpected internal error");
    return B2M_ERR_CUDA;
  }
}
