// Cross-GPU exchange over NVLink peer memory for the sequence-sharded path: a flag
// barrier between the ranks of one node and a gather of every rank's slice of an array.
// Peer pointers come from CUDA IPC mappings (dsalt_ipc_open); accesses are plain loads and
// stores (no multicast). Every wait is bounded (2 s of globaltimer) and reports to the
// device status word instead of hanging.
#include <algorithm>

#include "common.cuh"

namespace dsalt {

// rank `rank` publishes `epoch` in its own flag, then waits until every rank's flag has
// reached it. Writes made by this GPU before the call are visible to the peers after it.
// epoch <= 0: the epoch is own_flag[1] + 1, stored back in own_flag[1] (a device-side
// counter, so that a captured CUDA graph advances it on every replay).
__global__ void peer_barrier_kernel(int* own_flag, const int* const* flags, int n_ranks, int rank, int epoch_arg,
                                    int* err) {
  __shared__ int s_epoch;
  const int t = threadIdx.x;
  if (t == 0) {
    int epoch = epoch_arg;
    if (epoch <= 0) {
      epoch = own_flag[1] + 1;
      own_flag[1] = epoch;
    }
    s_epoch = epoch;
    __threadfence_system();
    *reinterpret_cast<volatile int*>(own_flag) = epoch;
    __threadfence_system();
  }
  __syncthreads();
  const int epoch = s_epoch;
  if (t < n_ranks && t != rank) {
    const volatile int* f = reinterpret_cast<const volatile int*>(flags[t]);
    const uint64_t t0 = globaltimer_ns();
    while (*f < epoch) {
      if (globaltimer_ns() - t0 > 2000000000ull) {
        report_device_error(err, 60);
        break;
      }
    }
    __threadfence_system();
  }
}

// dst[j * bytes, (j+1) * bytes) <- src[j][0, bytes) for every rank j != rank (16-byte units)
__global__ void peer_allgather_kernel(uint4* dst, const uint4* const* src, int n_ranks, int rank, int64_t n16) {
  const int j = blockIdx.y;
  if (j == rank) return;
  const uint4* s = src[j];
  uint4* d = dst + (int64_t)j * n16;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += (int64_t)gridDim.x * blockDim.x)
    d[i] = s[i];
}

int launch_peer_barrier(int* own_flag, const int* const* flags, int n_ranks, int rank, int epoch, int* err,
                        cudaStream_t stream) {
  if (n_ranks < 1 || n_ranks > 1024 || rank < 0 || rank >= n_ranks || !own_flag || !flags)
    return fail(DSALT_ERR_INVALID, "peer barrier: bad arguments");
  peer_barrier_kernel<<<1, n_ranks < 32 ? 32 : ((n_ranks + 31) / 32) * 32, 0, stream>>>(own_flag, flags, n_ranks,
                                                                                         rank, epoch, err);
  return check_cuda(cudaGetLastError(), "peer barrier launch");
}

int launch_peer_allgather(void* dst, const void* const* src, int n_ranks, int rank, int64_t bytes_per_rank,
                          cudaStream_t stream) {
  if (n_ranks < 1 || rank < 0 || rank >= n_ranks || !dst || !src || bytes_per_rank < 0)
    return fail(DSALT_ERR_INVALID, "peer allgather: bad arguments");
  if (bytes_per_rank % 16 || reinterpret_cast<uintptr_t>(dst) % 16)
    return fail(DSALT_ERR_INVALID, "peer allgather: 16-byte aligned slices required");
  if (bytes_per_rank == 0 || n_ranks == 1) return DSALT_OK;
  const int64_t n16 = bytes_per_rank / 16;
  const int64_t blocks = std::min<int64_t>((n16 + 255) / 256, 64);
  peer_allgather_kernel<<<dim3((unsigned)blocks, n_ranks), 256, 0, stream>>>(
      reinterpret_cast<uint4*>(dst), reinterpret_cast<const uint4* const*>(src), n_ranks, rank, n16);
  return check_cuda(cudaGetLastError(), "peer allgather launch");
}

int launch_peer_copy(void* dst, const void* src, int64_t bytes, cudaStream_t stream) {
  if (bytes < 0 || (bytes > 0 && (!dst || !src))) return fail(DSALT_ERR_INVALID, "peer copy: bad arguments");
  if (bytes == 0) return DSALT_OK;
  return check_cuda(cudaMemcpyAsync(dst, src, (size_t)bytes, cudaMemcpyDefault, stream), "peer copy");
}

}  // namespace dsalt
