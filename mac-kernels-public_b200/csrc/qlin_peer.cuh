// Output destinations in peer GPUs' memory and the flag protocol that orders the ranks' kernels.
//
// A sharded linear's epilogue stores each finished output tile straight into every rank's
// gathered activation buffer (plain 16-byte stores over NVLink to CUDA-IPC mappings; no multicast
// objects), so the all-gather of the output shards overlaps the GEMM tile by tile.
//
// Ordering between ranks uses one small pad per rank (PeerSync, in that rank's memory):
//   flags[src]  written by rank src (st.release.sys) with its launch count after each output-
//               writing kernel finished all its stores, in every rank's pad;
//   arrived     CTAs of the current output-writing kernel that finished (local);
//   epoch       output-writing kernels finished on this rank (local).
// A GEMM waits, before it reads any activation, until every rank's flag in its own pad reaches
// its own epoch: all ranks have finished the previous output-writing kernel, so (a) the slabs it
// is about to read are complete and (b) nobody still reads the buffer its epilogue will write.
// Every rank runs the same sequence of sharded linears, so epochs agree.  Epochs are counted on
// the device, which keeps the protocol valid under CUDA-graph replay.
//
// The wait is bounded (timeout_ms, default 10 s): on expiry the kernel records a status word,
// raises the CTA's abort flag and skips its tiles, so a missing rank shows up as an error code.
#pragma once
#include <cuda.h>

#include "qlin_ptx.cuh"

namespace qlin {

constexpr int kMaxPeers = 8;

struct PeerSync {
  unsigned int flags[kMaxPeers];
  unsigned int arrived;
  unsigned int epoch;
  unsigned int pad[6];
};
static_assert(sizeof(PeerSync) == 64, "PeerSync is one 64-byte pad");

// Tensor maps of the destinations (2-D {n, m} over each destination slab, box {128, 32}), for the
// TMA-store epilogue; a __grid_constant__ kernel parameter.
struct PeerMaps {
  CUtensorMap m[kMaxPeers];
};

struct PeerOut {
  int tma;       // 1: store each staged 32-token chunk with one TMA tensor store per destination
  int ndst;      // destinations of each output tile (0: plain per-element stores to GemmParams::y)
  int world;     // ranks taking part in the flag protocol (0: no waiting or signalling)
  int self;      // this rank's index in dst / sync
  int wait;      // wait for the previous output-writing kernel on every rank before reading X
  int signal;    // this kernel writes the output: publish the launch count when all CTAs finish
  unsigned int timeout_ms;
  PeerSync* own;               // this rank's pad (== sync[self])
  void* dst[kMaxPeers];        // per destination: base of this rank's output slab (row pitch ldy)
  PeerSync* sync[kMaxPeers];   // per rank: that rank's pad
};

__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// One thread: wait until every rank has published the epoch this rank has reached.  Returns false
// (recording the status word) when the wait runs out.
__device__ __forceinline__ bool peer_wait(const PeerOut& po, DeviceStatus* status, uint32_t site) {
  PeerSync* own = po.own;
  const unsigned int want = *reinterpret_cast<volatile unsigned int*>(&own->epoch);
  const uint64_t limit = (uint64_t)(po.timeout_ms ? po.timeout_ms : 10000u) * 1000000ull;
  const uint64_t t0 = globaltimer();
  for (int r = 0; r < po.world; ++r) {
    if (r == po.self || !qchk(BS_PEER_FLAG, r, kMaxPeers)) continue;
    while ((int)(ld_acquire_sys(&own->flags[r]) - want) < 0) {
      if (globaltimer() - t0 > limit) {
        if (status != nullptr && atomicExch(&status->timed_out, 1u) == 0u)
          status->where = (blockIdx.x << 8) | (site & 0xff);
        return false;
      }
      __nanosleep(128);
    }
  }
  return true;
}

// Thread 0 of each CTA, after a block barrier that follows all of the CTA's output stores: the
// last CTA to finish bumps this rank's epoch and publishes it in every rank's pad.
__device__ __forceinline__ void peer_signal_last_cta(const PeerOut& po) {
  PeerSync* own = po.own;
  __threadfence_system();
  const unsigned int total = gridDim.x * gridDim.y * gridDim.z;
  if (atomicAdd(&own->arrived, 1u) != total - 1) return;
  __threadfence_system();
  own->arrived = 0;
  const unsigned int e = own->epoch + 1;
  own->epoch = e;
#pragma unroll
  for (int r = 0; r < kMaxPeers; ++r)
    if (r < po.world && qchk(BS_PEER_FLAG, po.self, kMaxPeers)) st_release_sys(&po.sync[r]->flags[po.self], e);
}

}  // namespace qlin
