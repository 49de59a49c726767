// Host side of the tensor-parallel peer all-reduce (otf_ar_*) and its two standalone
// kernels: push (a rank's fp16 partial vector into every rank's receive buffer) and
// finish (wait for all ranks, sum, write fp16).  The fused forms live in the GEMV kernels
// (gemv2b.cu): o_proj / down_proj produce their rows straight into the buffers and the
// next grouped launch consumes them while staging its activation.
//
// No reference counterpart: the reference runs on one GPU; tensor parallelism over
// NVLink replaces the NCCL all_reduce that a row-parallel o_proj / down_proj needs.
#include <algorithm>
#include <cstring>

#include "tp_ar.cuh"

namespace otf {

__device__ int g_ar_device_error;  // set when a wait for peers gives up

constexpr int kArThreads = 256;
constexpr int64_t kArCtrlBytes = 4096;  // counters: epoch at 256*b, done at 256*b + 128

__global__ void __launch_bounds__(kArThreads) k_ar_push(const ArPeers* P, int b, const uint16_t* x, int n) {
  pdl_trigger();
  pdl_wait();
  const unsigned tag = ar_tag(P, b);
  for (int i = (int)(blockIdx.x * kArThreads + threadIdx.x); i < n; i += (int)(gridDim.x * kArThreads))
    ar_put(P, b, i, h2f(x[i]), tag);
}

__global__ void __launch_bounds__(kArThreads) k_ar_finish(const ArPeers* P, int b, uint16_t* out, int n) {
  pdl_trigger();
  pdl_wait();
  const unsigned tag = ar_tag(P, b);
  uint32_t budget = kArSpinLimit;
  int err = 0;
  const int n8 = n / 8;
  for (int v = (int)(blockIdx.x * kArThreads + threadIdx.x); v < n8; v += (int)(gridDim.x * kArThreads))
    reinterpret_cast<uint4*>(out)[v] = ar_sum8(P, b, 8 * (int64_t)v, tag, budget, err);
  if (blockIdx.x == 0)
    for (int i = 8 * n8 + (int)threadIdx.x; i < n; i += kArThreads) out[i] = ar_sum1(P, b, i, tag, budget, err);
  if (err) atomicExch(&g_ar_device_error, 1);
  __syncthreads();
  if (threadIdx.x == 0) ar_consumed(P, b);
}

int set_cuda_error(cudaError_t e);  // capi.cu
int check_device();                 // capi.cu

}  // namespace otf

struct otf_ar {
  int rank = 0, world = 0, dev = -1;
  int64_t max_elems = 0;
  size_t bytes = 0;
  void* local = nullptr;
  void* peer[otf::kArWorld] = {};
  bool opened = false;
  otf::ArPeers* d_peers = nullptr;
};

namespace otf {

// Errors raised by the waits of this file's kernels (the GEMV kernels keep their own flag).
int ar_device_error(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, otf::g_ar_device_error, sizeof(int)) != cudaSuccess) {
    set_cuda_error(cudaGetLastError());
    return -1;
  }
  if (clear && v) {
    const int z = 0;
    cudaMemcpyToSymbol(otf::g_ar_device_error, &z, sizeof(int));
  }
  return v;
}

// Device view of the peer table, for the fused GEMV forms.
const void* ar_device_table(const otf_ar* ar) { return ar && ar->opened ? ar->d_peers : nullptr; }
int ar_world(const otf_ar* ar) { return ar ? ar->world : 0; }
int64_t ar_max_elems(const otf_ar* ar) { return ar ? ar->max_elems : 0; }

}  // namespace otf

using otf::check_device;
using otf::set_cuda_error;

extern "C" OTF_API int otf_ar_create(int rank, int world, int64_t max_elems, void* ipc_handle, otf_ar** out) {
  if (!out || !ipc_handle || world < 1 || world > otf::kArWorld || rank < 0 || rank >= world || max_elems <= 0 ||
      max_elems > (int64_t)1 << 28)
    return OTF_ERR_INVALID;
  *out = nullptr;
  int st = check_device();
  if (st != OTF_OK) return st;
  otf_ar* ar = new otf_ar;
  ar->rank = rank;
  ar->world = world;
  ar->max_elems = otf::align_up(max_elems, 8);
  cudaGetDevice(&ar->dev);
  ar->bytes = (size_t)(otf::kArCtrlBytes + 2 * (int64_t)world * ar->max_elems * 8);
  cudaError_t e = cudaMalloc(&ar->local, ar->bytes);
  if (e == cudaSuccess) e = cudaMemset(ar->local, 0, ar->bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, ar->local);
  if (e != cudaSuccess) {
    if (ar->local) cudaFree(ar->local);
    delete ar;
    return set_cuda_error(e);
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == OTF_AR_HANDLE_BYTES, "IPC handle size");
  std::memcpy(ipc_handle, &h, sizeof(h));
  *out = ar;
  return OTF_OK;
}

extern "C" OTF_API int otf_ar_open(otf_ar* ar, const void* all_handles) {
  if (!ar || !all_handles || ar->opened) return OTF_ERR_INVALID;
  int dev = -1;
  cudaGetDevice(&dev);
  if (dev != ar->dev) return OTF_ERR_INVALID;
  const auto* hs = static_cast<const cudaIpcMemHandle_t*>(all_handles);
  cudaError_t e = cudaSuccess;
  int opened = 0;
  for (int r = 0; r < ar->world && e == cudaSuccess; ++r) {
    if (r == ar->rank) {
      ar->peer[r] = ar->local;
      continue;
    }
    e = cudaIpcOpenMemHandle(&ar->peer[r], hs[r], cudaIpcMemLazyEnablePeerAccess);
    if (e == cudaSuccess) ++opened;
  }
  otf::ArPeers t = {};
  if (e == cudaSuccess) {
    t.rank = ar->rank;
    t.world = ar->world;
    t.max_elems = ar->max_elems;
    for (int b = 0; b < 2; ++b) {
      for (int r = 0; r < ar->world; ++r) {
        char* base = static_cast<char*>(ar->peer[r]);
        t.data[b][r] = reinterpret_cast<unsigned long long*>(base + otf::kArCtrlBytes +
                                                             (int64_t)b * ar->world * ar->max_elems * 8);
      }
      t.epoch[b] = reinterpret_cast<unsigned*>(static_cast<char*>(ar->local) + 256 * b);
      t.done[b] = reinterpret_cast<unsigned*>(static_cast<char*>(ar->local) + 256 * b + 128);
    }
    e = cudaMalloc(&ar->d_peers, sizeof(t));
    if (e == cudaSuccess) e = cudaMemcpy(ar->d_peers, &t, sizeof(t), cudaMemcpyHostToDevice);
  }
  if (e != cudaSuccess) {
    for (int r = 0; r < ar->world; ++r)
      if (r != ar->rank && ar->peer[r]) cudaIpcCloseMemHandle(ar->peer[r]);
    for (int r = 0; r < ar->world; ++r) ar->peer[r] = nullptr;
    if (ar->d_peers) cudaFree(ar->d_peers);
    ar->d_peers = nullptr;
    (void)opened;
    return set_cuda_error(e);
  }
  ar->opened = true;
  return OTF_OK;
}

extern "C" OTF_API int otf_ar_destroy(otf_ar* ar) {
  if (!ar) return OTF_ERR_INVALID;
  int dev = -1;
  cudaGetDevice(&dev);
  if (dev != ar->dev) cudaSetDevice(ar->dev);
  cudaDeviceSynchronize();
  for (int r = 0; r < ar->world; ++r)
    if (r != ar->rank && ar->peer[r]) cudaIpcCloseMemHandle(ar->peer[r]);
  if (ar->d_peers) cudaFree(ar->d_peers);
  if (ar->local) cudaFree(ar->local);
  if (dev != ar->dev && dev >= 0) cudaSetDevice(dev);
  delete ar;
  return OTF_OK;
}

static int ar_launch_blocks(int64_t n) {
  return (int)std::max<int64_t>(1, std::min<int64_t>(otf::ceil_div((int)n, 2048), 64));
}

extern "C" OTF_API int otf_ar_push(otf_ar* ar, int buf, const void* x, int64_t n, void* stream) {
  if (!ar || !ar->opened || !x || (buf != 0 && buf != 1) || n <= 0 || n > ar->max_elems) return OTF_ERR_INVALID;
  int st = check_device();
  if (st != OTF_OK) return st;
  return set_cuda_error(otf::launch_pdl(otf::k_ar_push, dim3(ar_launch_blocks(n)), dim3(otf::kArThreads), 0,
                                        static_cast<cudaStream_t>(stream), 1u,
                                        static_cast<const otf::ArPeers*>(ar->d_peers), buf,
                                        static_cast<const uint16_t*>(x), (int)n));
}

extern "C" OTF_API int otf_ar_finish(otf_ar* ar, int buf, void* out, int64_t n, void* stream) {
  if (!ar || !ar->opened || !out || (buf != 0 && buf != 1) || n <= 0 || n > ar->max_elems) return OTF_ERR_INVALID;
  if (reinterpret_cast<uintptr_t>(out) % 16) return OTF_ERR_INVALID;
  int st = check_device();
  if (st != OTF_OK) return st;
  return set_cuda_error(otf::launch_pdl(otf::k_ar_finish, dim3(ar_launch_blocks(n)), dim3(otf::kArThreads), 0,
                                        static_cast<cudaStream_t>(stream), 1u,
                                        static_cast<const otf::ArPeers*>(ar->d_peers), buf,
                                        static_cast<uint16_t*>(out), (int)n));
}
