// Reduced cross-entropy for callers that cannot allocate device memory.
//
// b2k_cross_entropy_mean_noalloc computes the same result as the allocating
// sequence b2k_cross_entropy (fp32 row losses) -> b2k_ce_reduce -> b2k_ce_mean,
// but its intermediate storage (the per-row losses and the fp64 [sum, count]
// pair) is a fixed buffer compiled into this library instead of memory the
// caller passes in.  It exists for hosts that cannot hand out scratch: a
// process whose device memory is entirely owned and pre-reserved by another
// runtime (a serving engine or a framework allocator that must account for
// every byte), or a foreign-function binding that has device pointers for its
// inputs and outputs but no allocator to call.
//
// The buffer is a file-scope __device__ array, so every GPU that loads the
// library holds it (1 MiB + 256 B) until the process exits.  Host code cannot
// use the array's name as a device address (in host code it names a host-side
// stand-in); the device address is obtained once per device with
// cudaGetSymbolAddress, with that device current, on the first call made on
// that device.  Make that first call before any stream capture.  The cached
// address belongs to the device's context at that first call: a process that
// resets a device (cudaDeviceReset) must not call this entry point on that
// device afterwards, because the cached address is not looked up again.  All
// calls
// share the one buffer: two calls whose work overlaps on the GPU (different
// streams, or different host threads on the same device) race and give wrong
// results.  Nothing in the buffer needs clearing between calls: every row
// loss and both halves of the pair are rewritten by each call.
#include <mutex>

#include "common.cuh"

namespace {

constexpr int64_t kNoallocMaxRows = B2K_NOALLOC_MAX_ROWS;
constexpr size_t kLossBytes = (size_t)kNoallocMaxRows * sizeof(float);  // 1 MiB

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_dev_ptr[kMaxDevices] = {nullptr};

}  // namespace

// [0, 1 MiB): per-row fp32 losses; [1 MiB, +16): the fp64 (sum, count) pair
static __device__ __align__(256) unsigned char g_noalloc_scratch[kLossBytes + 256];

extern "C" int b2k_cross_entropy_mean_noalloc(const void* x, int64_t ldx, const int64_t* tgt,
                                              int64_t M, int64_t N, int dtype,
                                              int64_t ignore_index, float* out, void* stream) {
  if (M > kNoallocMaxRows) {
    b2k::set_error(
        "b2k_cross_entropy_mean_noalloc: %lld rows exceed the built-in scratch of %lld rows; "
        "use b2k_cross_entropy + b2k_ce_reduce + b2k_ce_mean with caller scratch",
        (long long)M, (long long)kNoallocMaxRows);
    return B2K_EINVAL;
  }
  B2K_REQUIRE(M >= 0 && N >= 0, "b2k_cross_entropy_mean_noalloc: negative shape");
  B2K_REQUIRE(out != nullptr, "b2k_cross_entropy_mean_noalloc: null output");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    b2k::set_error("b2k_cross_entropy_mean_noalloc: cudaGetDevice failed: %s",
                   cudaGetErrorString(e));
    return B2K_ELAUNCH;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    b2k::set_error("b2k_cross_entropy_mean_noalloc: device %d outside the %d devices this "
                   "entry point keeps scratch addresses for", dev, kMaxDevices);
    return B2K_EINVAL;
  }
  void* base;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_dev_ptr[dev] == nullptr) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess || p == nullptr) {
        b2k::set_error("b2k_cross_entropy_mean_noalloc: cudaGetSymbolAddress failed: %s",
                       cudaGetErrorString(e));
        return B2K_ELAUNCH;
      }
      g_dev_ptr[dev] = p;
    }
    base = g_dev_ptr[dev];
  }
  float* row_loss = static_cast<float*>(base);
  double* sumcount = reinterpret_cast<double*>(static_cast<unsigned char*>(base) + kLossBytes);
  int st = b2k_cross_entropy(x, ldx, tgt, row_loss, M, N, dtype, B2K_F32, ignore_index, stream);
  if (st != B2K_OK) return st;
  st = b2k_ce_reduce(row_loss, tgt, M, ignore_index, sumcount, stream);
  if (st != B2K_OK) return st;
  return b2k_ce_mean(sumcount, out, stream);
}
