// pk_noalloc.cu -- a host-pointer softmax that allocates no memory.
//
// The drop-in pk_softmax_rows copies the caller's rows into a device
// workspace it grows with cudaMalloc. Some callers cannot let a library
// allocate: a real-time audio callback that must not block on the allocator
// (cudaMalloc can synchronise the device and take milliseconds), or a process
// whose device memory is carved up in advance by its own pool, so that any
// allocation outside that pool fails or steals from it. pk_softmax_rows_noalloc
// does the same work with its staging buffer in a fixed array that is part of
// the library image: PK_NOALLOC_MAX_FLOATS floats (16 MiB) on every device
// that loads the library, held until the process exits.
//
// Set-up: the first call on a device looks up the array's device address
// (cudaGetSymbolAddress, with that device current) and caches it per device
// index; make that first call before any stream capture. The cache does not
// survive cudaDeviceReset (the module is loaded again and the array may move):
// a process that resets a device must not call this entry point afterwards.
// Later calls only copy, launch and synchronise on the per-thread default
// stream.
//
// The array is shared by every call on a device and keeps the last call's
// contents (each call overwrites what it uses). Calls whose GPU work overlaps
// -- e.g. from two host threads at once -- race on it.
#include <mutex>

#include "pk_common.cuh"

#define PK_NOALLOC_MAX_FLOATS (4u << 20)

static __device__ __align__(256) float g_noalloc_scratch[PK_NOALLOC_MAX_FLOATS];

static std::mutex g_noalloc_setup;
#define PK_NOALLOC_MAX_DEVICES 64
static float *g_noalloc_ptr[PK_NOALLOC_MAX_DEVICES];

// Device address of the scratch array on the current device (set-up on first use).
static int noalloc_scratch(float **out) {
  int dev = -1;
  const cudaError_t de = cudaGetDevice(&dev);
  if (de != cudaSuccess) {
    cudaGetLastError();
    return pkcu_fail(PKCU_ERR_CUDA, "pk_softmax_rows_noalloc: cudaGetDevice: %s",
                     cudaGetErrorString(de));
  }
  if (dev < 0 || dev >= PK_NOALLOC_MAX_DEVICES)
    return pkcu_fail(PKCU_ERR_ARG, "pk_softmax_rows_noalloc: device index %d (at most %d devices)",
                     dev, PK_NOALLOC_MAX_DEVICES);
  std::lock_guard<std::mutex> lock(g_noalloc_setup);
  if (!g_noalloc_ptr[dev]) {
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      cudaGetLastError();
      return pkcu_fail(PKCU_ERR_CUDA, "pk_softmax_rows_noalloc: cudaGetSymbolAddress: %s",
                       cudaGetErrorString(e));
    }
    g_noalloc_ptr[dev] = static_cast<float *>(p);
  }
  *out = g_noalloc_ptr[dev];
  return PKCU_OK;
}

extern "C" int pk_softmax_rows_noalloc(float *x, int n_rows, int len) {
  if (n_rows < 0 || len < 0) return pkcu_fail(PKCU_ERR_ARG, "pk_softmax_rows_noalloc: bad argument");
  if (n_rows == 0 || len == 0) return PKCU_OK;   // nothing to do: x may be NULL, as for the drop-ins
  if (!x) return pkcu_fail(PKCU_ERR_ARG, "pk_softmax_rows_noalloc: NULL x");
  const unsigned long long n = (unsigned long long)n_rows * (unsigned long long)len;
  if (n > PK_NOALLOC_MAX_FLOATS)
    return pkcu_fail(PKCU_ERR_ARG,
                     "pk_softmax_rows_noalloc: %llu floats exceed the %u-float static buffer", n,
                     PK_NOALLOC_MAX_FLOATS);
  float *d = nullptr;
  int st = noalloc_scratch(&d);
  if (st) return st;
  const cudaStream_t s = cudaStreamPerThread;
  const size_t bytes = (size_t)n * sizeof(float);
  if (cudaMemcpyAsync(d, x, bytes, cudaMemcpyHostToDevice, s) != cudaSuccess)
    return pkcu_fail(PKCU_ERR_CUDA, "pk_softmax_rows_noalloc: %s", cudaGetErrorString(cudaGetLastError()));
  st = pkcu_softmax_rows(d, n_rows, len, s);
  if (st) {
    cudaStreamSynchronize(s);
    return st;
  }
  if (cudaMemcpyAsync(x, d, bytes, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return pkcu_fail(PKCU_ERR_CUDA, "pk_softmax_rows_noalloc: %s", cudaGetErrorString(cudaGetLastError()));
  return PKCU_OK;
}
