// Peer memory across the GPUs of one node: buffers that every rank maps, and a
// bounded device-side barrier over them.
//
// The view-parallel step keeps one process per GPU.  Buffers created with
// vs_peer_alloc are plain cudaMalloc allocations whose CUDA IPC handles the
// ranks exchange (through torch.distributed); vs_peer_open maps a peer's
// buffer into this process, after which this GPU's kernels load and store it
// directly over NVLink.  vs_peer_barrier orders the ranks' streams: every rank
// stores the barrier epoch into its slot of every peer's flag array (a
// system-scope release after a system fence), then waits until all slots of
// its own array carry the epoch, for two seconds at most.  A wait that runs
// out sets VS_DERR_WAIT in the ctx's device error word (read by vs_ctx_check
// and by the next count readback) and returns; it never traps.
#include <string.h>

#include "vs_internal.cuh"

namespace {

constexpr uint64_t BARRIER_WAIT_NS = 2000000000ull;  // give up after two seconds
constexpr uint32_t BARRIER_SPIN_LIMIT = 1u << 26;    // backstop on the iteration count

struct FlagPtrs {
  uint32_t* f[VS_PEER_MAX];
};

__device__ __forceinline__ void store_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t load_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Thread r signals peer r and then waits for peer r's signal.
__global__ void peer_barrier_kernel(FlagPtrs flags, uint32_t rank, uint32_t world, uint32_t epoch, uint32_t* err) {
  const uint32_t r = threadIdx.x;
  if (r >= world) return;
  __threadfence_system();
  store_release_sys(flags.f[r] + rank, epoch);
  const uint32_t* mine = flags.f[rank] + r;
  const uint64_t t0 = global_ns();
  for (uint32_t spins = 0;; ++spins) {
    if ((int32_t)(load_acquire_sys(mine) - epoch) >= 0) break;
    if (spins >= BARRIER_SPIN_LIMIT || global_ns() - t0 > BARRIER_WAIT_NS) {
      atomicOr(err, VS_DERR_WAIT);
      break;
    }
    __nanosleep(128);
  }
  __threadfence_system();
}

}  // namespace

extern "C" {

VS_API vs_status vs_peer_alloc(vs_ctx* ctx, uint64_t bytes, void** dev_ptr, vs_ipc_handle* handle) {
  if (!ctx) return VS_ERR_INVALID;
  if (!dev_ptr || !handle || bytes == 0) return vs_fail(ctx, VS_ERR_INVALID, "peer_alloc: bad arguments");
  VS_CUDA(ctx, cudaSetDevice(ctx->device));
  void* p = nullptr;
  VS_CUDA(ctx, cudaMalloc(&p, bytes));
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return vs_cuda(ctx, e, "cudaIpcGetMemHandle");
  }
  static_assert(sizeof(h) <= sizeof(handle->bytes), "IPC handle size");
  memset(handle->bytes, 0, sizeof(handle->bytes));
  memcpy(handle->bytes, &h, sizeof(h));
  *dev_ptr = p;
  return VS_OK;
}

VS_API vs_status vs_peer_free(vs_ctx* ctx, void* dev_ptr) {
  if (!ctx) return VS_ERR_INVALID;
  if (!dev_ptr) return VS_OK;
  VS_CUDA(ctx, cudaSetDevice(ctx->device));
  return vs_cuda(ctx, cudaFree(dev_ptr), "peer_free");
}

VS_API vs_status vs_peer_open(vs_ctx* ctx, const vs_ipc_handle* handle, void** dev_ptr) {
  if (!ctx) return VS_ERR_INVALID;
  if (!handle || !dev_ptr) return vs_fail(ctx, VS_ERR_INVALID, "peer_open: bad arguments");
  VS_CUDA(ctx, cudaSetDevice(ctx->device));
  cudaIpcMemHandle_t h;
  memcpy(&h, handle->bytes, sizeof(h));
  return vs_cuda(ctx, cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
}

VS_API vs_status vs_peer_close(vs_ctx* ctx, void* dev_ptr) {
  if (!ctx) return VS_ERR_INVALID;
  if (!dev_ptr) return VS_OK;
  VS_CUDA(ctx, cudaSetDevice(ctx->device));
  return vs_cuda(ctx, cudaIpcCloseMemHandle(dev_ptr), "cudaIpcCloseMemHandle");
}

VS_API vs_status vs_peer_barrier(vs_ctx* ctx, uint32_t* const* peer_flags, uint32_t world, uint32_t rank,
                                 uint32_t epoch) {
  if (!ctx) return VS_ERR_INVALID;
  if (!peer_flags || world == 0 || world > VS_PEER_MAX || rank >= world)
    return vs_fail(ctx, VS_ERR_INVALID, "peer_barrier: world %u rank %u", world, rank);
  FlagPtrs f{};
  for (uint32_t r = 0; r < world; ++r) {
    if (!peer_flags[r]) return vs_fail(ctx, VS_ERR_INVALID, "peer_barrier: null flags of rank %u", r);
    f.f[r] = peer_flags[r];
  }
  peer_barrier_kernel<<<1, 32, 0, ctx->stream>>>(f, rank, world, epoch, ctx->d_err); ++ctx->launches;
  return vs_cuda(ctx, cudaGetLastError(), "peer_barrier launch");
}

VS_API vs_status vs_ctx_check(vs_ctx* ctx) {
  if (!ctx) return VS_ERR_INVALID;
  return vs_check_device_error(ctx, "device");
}

}  // extern "C"
