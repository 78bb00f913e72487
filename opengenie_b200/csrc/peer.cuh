// Cross-GPU barrier for the sequence-parallel exchange over NVLink.
//
// Every rank keeps a block of 16 32-bit words in its own memory, mapped into the
// other ranks' address spaces (CUDA IPC): words [0, 8) are arrival slots, one
// per rank; word 8 counts the barriers this rank has passed.  Barrier number
// e = count + 1 (the same sequence on every rank, since all ranks run the same
// barriers in the same order): rank r stores e into slot r of every peer's block
// with a system-scope release, waits until every peer has stored at least e
// into its own slot of r's block (system-scope acquire), then advances its
// count.  Keeping the count in device memory makes the kernel's arguments the
// same on every call, so a step that contains barriers can be captured once in
// a CUDA graph and replayed.  The producing kernels fence their peer stores
// system-wide before they exit, and this kernel runs after them on the same
// stream, so data written to a peer is visible there once the peer passes the
// barrier.  The wait is bounded: past the limit it records OGX_ERR_TIMEOUT in
// the device status word and returns (the host reads the status; nothing hangs).
#pragma once

#include "ogx_sm100.cuh"

namespace ogx {

struct PeerSignals {
  unsigned int* slot[8];  // peer p's signal array (slot[rank] is the local one)
};

constexpr int kPeerSignalWords = 16;
constexpr int kPeerCountWord = 8;

__global__ void __launch_bounds__(32) peer_barrier_kernel(unsigned int* local, PeerSignals peers, int rank,
                                                          int world) {
  pdl_trigger();
  pdl_wait();  // the producing kernel has completed (its peer stores were fenced system-wide)
  const int i = threadIdx.x;
  const unsigned int epoch = *reinterpret_cast<volatile unsigned int*>(local + kPeerCountWord) + 1u;
  if (i < world && i != rank) {
    // constant-index selects: a runtime index into the parameter array would copy it to local memory
    unsigned int* peer = peers.slot[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) peer = (i == j) ? peers.slot[j] : peer;
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(peer + rank), "r"(epoch) : "memory");
    const unsigned long long t0 = global_ns();
    for (uint32_t n = 0;; ++n) {
      unsigned int v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(local + i) : "memory");
      if (static_cast<int>(v - epoch) >= 0) break;
      if ((n & 255u) == 255u && global_ns() - t0 > kWaitLimitNs) {
        atomicOr(&g_ogx_status, OGX_ERR_TIMEOUT);
        break;
      }
    }
  }
  __syncwarp();  // every lane has read the count
  if (i == 0) local[kPeerCountWord] = epoch;
}

// The barrier of ogx_peer_barrier_static, for ranks that are GPUs of one process.  Its arrival slots are
// page-locked host memory mapped into every GPU of the process: slots[d * kPeerSignalWords + r] holds the
// latest barrier number rank r announced to device d.  No GPU reads or writes another GPU's memory; the
// barrier count stays in this GPU's own block (`local`).  Stores go out with a system-scope release, loads
// come in with a system-scope acquire; the wait is bounded as in peer_barrier_kernel.
struct DeviceList {
  int d[8];  // rank i's device ordinal
};

__device__ __forceinline__ int device_of(const DeviceList& devs, int i) {
  int d = devs.d[0];  // constant-index selects (a runtime index into the parameter array would go to local memory)
#pragma unroll
  for (int j = 1; j < 8; ++j) d = (i == j) ? devs.d[j] : d;
  return d;
}

__global__ void __launch_bounds__(32) host_slot_barrier_kernel(unsigned int* local, unsigned int* slots,
                                                               DeviceList devs, int rank, int world) {
  pdl_trigger();
  pdl_wait();
  const int i = threadIdx.x;
  const unsigned int epoch = *reinterpret_cast<volatile unsigned int*>(local + kPeerCountWord) + 1u;
  if (i < world && i != rank) {
    unsigned int* to_peer = slots + device_of(devs, i) * kPeerSignalWords + rank;
    unsigned int* from_peer = slots + device_of(devs, rank) * kPeerSignalWords + i;
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(to_peer), "r"(epoch) : "memory");
    const unsigned long long t0 = global_ns();
    for (uint32_t n = 0;; ++n) {
      unsigned int v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(from_peer) : "memory");
      if (static_cast<int>(v - epoch) >= 0) break;
      if ((n & 255u) == 255u && global_ns() - t0 > kWaitLimitNs) {
        atomicOr(&g_ogx_status, OGX_ERR_TIMEOUT);
        break;
      }
    }
  }
  __syncwarp();  // every lane has read the count
  if (i == 0) local[kPeerCountWord] = epoch;
}

}  // namespace ogx
