// Max-reduction of one fp32 value over the ranks of a sequence split, through NVLink peer memory.
//
// Replaces the 4-byte NCCL all-reduce (MAX) that the sequence-split step makes at every FP8
// quantisation point (six per block: the three norm outputs, the two attention outputs and the FF
// hidden; the split module's all_reduce_max). Each rank owns a mailbox in its own GPU memory,
// allocated here and shared with the other ranks of the node through CUDA IPC handles:
//   box[sender * SA3_PEER_SLOTS + slot]  (uint64: epoch << 32 | fp32 bits), then one uint64 epoch counter.
// One exchange is one warp on one SM: lane 0 takes the next epoch e from the counter; lane s < world
// stores (e, value) into slot e % SA3_PEER_SLOTS, row `rank`, of rank s's mailbox (st.release.sys over
// NVLink), then waits (ld.acquire.sys, bounded) until row s of its own mailbox carries epoch e; the
// maximum of the world values replaces the local value. Every rank makes the same exchanges in the same
// order, so the epochs agree. A rank can be at most one exchange ahead of the slowest rank (it needs
// everyone's word of the current epoch to finish), so with 4 slots a word is never overwritten before
// it is read. The wait gives up after SA3_WAIT_BUDGET_CYCLES (about a second), records a device error
// (site 90) and keeps the local value.
// Requirements (the caller checks them): every rank on its own GPU of one node, with peer access between
// them; kernels that wait on each other are never launched on one GPU.
#include <cuda_runtime.h>

#include <cstring>

#include "common.cuh"
#include "host_util.h"

namespace sa3 {
SA3_DEFINE_ERROR_READER(read_error_peer)

struct PeerBoxes {
  unsigned long long* box[SA3_PEER_MAX_RANKS];
};

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(32, 1) peer_max_kernel(float* value, PeerBoxes pb, int rank, int world) {
  grid_dep_wait();
  const int lane = threadIdx.x;
  unsigned long long* mine = pb.box[rank];
  unsigned long long* counter = mine + SA3_PEER_MAX_RANKS * SA3_PEER_SLOTS;
  unsigned int e = 0;
  if (lane == 0) {
    e = (unsigned int)(*counter) + 1u;
    *counter = e;
  }
  e = __shfl_sync(0xffffffffu, e, 0);
  const float v = *value;
  const int slot = (int)(e % SA3_PEER_SLOTS);
  const unsigned long long word = ((unsigned long long)e << 32) | __float_as_uint(v);
  float m = v;
  bool ok = true;
  if (lane < world) {
    st_release_sys(pb.box[lane] + rank * SA3_PEER_SLOTS + slot, word);
    const unsigned long long* src = mine + lane * SA3_PEER_SLOTS + slot;
    unsigned long long w = ld_acquire_sys(src);
    const long long t0 = clock64();
    while ((unsigned int)(w >> 32) != e) {
      if (clock64() - t0 > SA3_WAIT_BUDGET_CYCLES) {
        ok = false;
        break;
      }
      __nanosleep(32);
      w = ld_acquire_sys(src);
    }
    if (ok) m = fmaxf(m, __uint_as_float((unsigned int)(w & 0xffffffffull)));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const bool all_ok = __all_sync(0xffffffffu, ok);
  if (lane == 0) {
    if (all_ok)
      *value = m;
    else
      record_error(SA3_DEVERR_TIMEOUT, 90);
  }
}

}  // namespace sa3

using namespace sa3;

extern "C" int sa3_peer_box_bytes(void) {
  return (int)((SA3_PEER_MAX_RANKS * SA3_PEER_SLOTS + 1) * sizeof(unsigned long long));
}

extern "C" int sa3_peer_box_alloc(void** box) {
  if (!box) return SA3_ERR_ARG;
  void* p = nullptr;
  const size_t bytes = (size_t)sa3_peer_box_bytes();
  if (cudaMalloc(&p, bytes) != cudaSuccess) return SA3_ERR_LAUNCH;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(p);
    return SA3_ERR_LAUNCH;
  }
  *box = p;
  return SA3_OK;
}

extern "C" int sa3_peer_box_free(void* box) {
  if (!box) return SA3_ERR_ARG;
  return cudaFree(box) == cudaSuccess ? SA3_OK : SA3_ERR_LAUNCH;
}

extern "C" int sa3_ipc_handle_bytes(void) { return (int)sizeof(cudaIpcMemHandle_t); }

extern "C" int sa3_ipc_get_handle(void* ptr, void* handle) {
  if (!ptr || !handle) return SA3_ERR_ARG;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, ptr) != cudaSuccess) return SA3_ERR_LAUNCH;
  memcpy(handle, &h, sizeof(h));
  return SA3_OK;
}

extern "C" int sa3_ipc_open_handle(const void* handle, void** ptr) {
  if (!handle || !ptr) return SA3_ERR_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return SA3_ERR_LAUNCH;
  *ptr = p;
  return SA3_OK;
}

extern "C" int sa3_ipc_close_handle(void* ptr) {
  if (!ptr) return SA3_ERR_ARG;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? SA3_OK : SA3_ERR_LAUNCH;
}

extern "C" int sa3_peer_max(float* value, void* const* boxes, int rank, int world, void* stream) {
  if (!value || !boxes || world < 1 || world > SA3_PEER_MAX_RANKS || rank < 0 || rank >= world) return SA3_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(value) & 3) return SA3_ERR_ALIGN;
  PeerBoxes pb;
  for (int i = 0; i < SA3_PEER_MAX_RANKS; ++i) {
    pb.box[i] = i < world ? static_cast<unsigned long long*>(boxes[i]) : nullptr;
    if (i < world && (!pb.box[i] || (reinterpret_cast<uintptr_t>(pb.box[i]) & 7))) return SA3_ERR_ARG;
  }
  launch_ex(peer_max_kernel, dim3(1), dim3(32), 0, reinterpret_cast<cudaStream_t>(stream), 1, value, pb, rank, world);
  return launch_status();
}
