// Symmetric memory across the GPUs of one node (one process per GPU).
//
// Every rank allocates a buffer of the same size; CUDA IPC handles are
// exchanged over the process group (host side, Python) and each rank maps its
// peers' buffers, giving a table of device pointers that kernels use for
// direct NVLink loads and stores. A region of each buffer holds signal pads:
// 32-bit counters that peers increment with release semantics after writing
// data, and that the owner polls with acquire semantics - always with a
// %globaltimer bound (b200::kWaitLimitNs), after which the kernel records
// kErrPeerWait in the status word and carries on, so a missing peer can never
// hang the GPU.
//
// The reference has no communication backend (collectives are closures
// injected by an external runtime, TensorParallelSwitchLinear.swift:56-74);
// this is the B200 replacement that the fused collective kernels build on.
#include "b200_common.cuh"
#include "b200_comm.cuh"

extern "C" {

// Allocate `bytes` of zeroed device memory and export its IPC handle
// (64 bytes written to handle_out).
int b200_symm_alloc(size_t bytes, void** ptr, void* handle_out) {
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) return (int)e;
  e = cudaMemset(*ptr, 0, bytes);
  if (e != cudaSuccess) return (int)e;
  e = cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t*>(handle_out), *ptr);
  return (int)e;
}

// Map a peer's buffer from its IPC handle.
int b200_symm_open(const void* handle, void** peer_ptr) {
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return (int)cudaIpcOpenMemHandle(peer_ptr, h, cudaIpcMemLazyEnablePeerAccess);
}

int b200_symm_close(void* peer_ptr) { return (int)cudaIpcCloseMemHandle(peer_ptr); }
int b200_symm_free(void* ptr) { return (int)cudaFree(ptr); }
int b200_ipc_handle_size() { return (int)sizeof(cudaIpcMemHandle_t); }

}  // extern "C"

namespace b200 {

// Test kernel: every rank adds 1 to slot [rank] of every peer's pad, then
// waits for all peers' increments on its own pad (bounded). status[0] = 1 on
// success, 0 on timeout.
__global__ void signal_roundtrip_kernel(CommCtx ctx, int pad, int* status) {
  if (threadIdx.x != 0) return;
  for (int j = 0; j < ctx.world; ++j) signal_add(ctx.pad_ptr(j, pad, ctx.rank), 1u);
  bool ok = true;
  for (int j = 0; j < ctx.world; ++j) ok &= wait_counter(ctx.pad_ptr(ctx.rank, pad, j), ctx.expect(pad, j) + 1u);
  for (int j = 0; j < ctx.world; ++j) ctx.bump(pad, j, 1u);
  status[0] = ok ? 1 : 0;
}

}  // namespace b200

extern "C" int b200_comm_signal_roundtrip(const void* ctx_bytes, int pad, int* status, cudaStream_t st) {
  b200::CommCtx ctx;
  memcpy(&ctx, ctx_bytes, sizeof(ctx));
  b200::signal_roundtrip_kernel<<<1, 32, 0, st>>>(ctx, pad, status);
  return (int)cudaGetLastError();
}

extern "C" int b200_comm_ctx_size() { return (int)sizeof(b200::CommCtx); }

B200_STATUS_ACCESSORS(symm)
