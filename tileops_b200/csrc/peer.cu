// Rank barrier on the GPU for the processes of one node, over memory mapped with CUDA IPC:
// the completion step of the gathering GEMMs (to_awq_gemm_gather), whose kernels store each
// rank's output slice into every rank's buffer. Instead of a collective per layer, each rank
// runs one tiny kernel after its GEMM: it raises its slot in every rank's flag array to the
// next barrier count (a release store at system scope, after the GEMM's own system-scope
// fence), then waits until every rank's slot in its own array has reached that count (acquire
// loads). Work queued after it on the stream therefore reads peer data that is complete.
//
// The count lives in device memory and advances in the kernel itself, so a CUDA graph that
// captured the barrier replays it correctly; every rank must run the same sequence of
// barriers. Waits are bounded: after the library's wait limit the kernel records a timeout in
// the device error word and returns (a rank that left, or one that never launched its part).
//
// With launch overlap on, the barrier is launched as a programmatic dependent of the GEMM: it
// is resident before the GEMM ends and starts at griddepcontrol.wait (the GEMM complete, its
// stores visible), then lets the next kernel in the stream launch at once, so that kernel's
// weight stream, which reads nothing the ranks exchange, overlaps the flag round trip; the
// next kernel's own griddepcontrol.wait still waits for this barrier to finish.
#include "common.cuh"
#include "sm100.cuh"

namespace tob {
namespace {

constexpr int kPeerMax = 8;
struct PeerFlags {
  unsigned long long* f[kPeerMax];  // rank r's flag array (kPeerMax slots), mapped here
};

__global__ void __launch_bounds__(32) k_peer_barrier(PeerFlags flags, int world, int rank,
                                                     unsigned long long* counter, int* err) {
  const int lane = threadIdx.x;
  grid_dependency_wait();
  grid_dependents_launch();
  unsigned long long target = 0;
  if (lane == 0) {
    target = *counter + 1;
    *counter = target;
  }
  target = __shfl_sync(0xffffffffu, target, 0);
  if (lane < world) {
    unsigned long long* slot = flags.f[lane] + rank;
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(slot), "l"(target) : "memory");
    const unsigned long long* mine = flags.f[rank] + lane;
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(mine) : "memory");
    if (v < target) {
      const uint64_t t0 = sm100::globaltimer_ns();
      while (true) {
        asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(mine) : "memory");
        if (v >= target) break;
        if (sm100::globaltimer_ns() - t0 > sm100::kWaitLimitNs) {
          if (err) atomicExch(err, (int)kErrWaitTimeout);
          break;
        }
      }
    }
  }
  __syncwarp();
}

}  // namespace
}  // namespace tob

extern "C" {

size_t to_peer_flags_bytes(void) { return tob::kPeerMax * sizeof(unsigned long long); }

int to_peer_barrier(unsigned long long* const* flag_ranks, int world, int rank,
                    unsigned long long* counter, void* stream) {
  if (world < 1 || world > tob::kPeerMax || rank < 0 || rank >= world)
    return tob::fail(TO_EINVAL, "to_peer_barrier: rank %d of %d (1 to %d ranks)", rank, world,
                     tob::kPeerMax);
  if (!flag_ranks || !counter) return tob::fail(TO_EINVAL, "to_peer_barrier: null argument");
  tob::PeerFlags f = {};
  for (int r = 0; r < world; ++r) {
    if (!flag_ranks[r]) return tob::fail(TO_EINVAL, "to_peer_barrier: null flags of rank %d", r);
    f.f[r] = flag_ranks[r];
  }
  int* err = tob::device_error_ptr();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1, 1, 1);
  cfg.blockDim = dim3(32, 1, 1);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  if (tob::launch_overlap()) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  const cudaError_t e = cudaLaunchKernelEx(&cfg, tob::k_peer_barrier, f, world, rank, counter, err);
  if (e != cudaSuccess) return tob::cuda_fail(e, "to_peer_barrier launch");
  return tob::check_launch("to_peer_barrier");
}

}  // extern "C"
