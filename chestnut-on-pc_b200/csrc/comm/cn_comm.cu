// Clip-end result gather over NCCL (libcncomm.so; include/chestnut_comm.h).
//
// One communicator per process/GPU.  Init and the gather run NCCL in
// non-blocking mode and poll with a wall-clock limit, so a rank that never
// arrives turns into CN_COMM_ERR_TIMEOUT (and an aborted communicator) rather
// than a hang.  The gather moves host f64 buffers through a device staging
// buffer owned by the communicator.
#include <cuda_runtime.h>
#include <nccl.h>

#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <thread>

#include "../../../include/chestnut_comm.h"

struct cn_comm {
  ncclComm_t comm = nullptr;
  cudaStream_t stream = nullptr;
  int device = 0, nranks = 0, rank = 0;
  double* dbuf = nullptr;  // [nranks + 1][cap] doubles: gathered rows, then this rank's send row
  size_t cap = 0;
  bool aborted = false;
};

namespace {
thread_local char g_err[512] = "";

void set_err(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

using Clock = std::chrono::steady_clock;

// Poll a non-blocking NCCL call to completion (ncclSuccess) or failure.
int wait_comm(cn_comm* c, int timeout_ms, const char* what) {
  const auto t0 = Clock::now();
  while (true) {
    ncclResult_t st = ncclSuccess;
    ncclResult_t r = ncclCommGetAsyncError(c->comm, &st);
    if (r != ncclSuccess) {
      set_err("%s: ncclCommGetAsyncError: %s", what, ncclGetErrorString(r));
      return CN_COMM_ERR_NCCL;
    }
    if (st == ncclSuccess) return 0;
    if (st != ncclInProgress) {
      set_err("%s: %s", what, ncclGetErrorString(st));
      return CN_COMM_ERR_NCCL;
    }
    if (std::chrono::duration_cast<std::chrono::milliseconds>(Clock::now() - t0).count() > timeout_ms) {
      set_err("%s: no progress within %d ms (a rank did not arrive)", what, timeout_ms);
      return CN_COMM_ERR_TIMEOUT;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
}

// Wait for the communicator's stream, watching for NCCL errors.
int wait_stream(cn_comm* c, int timeout_ms, const char* what) {
  const auto t0 = Clock::now();
  while (true) {
    cudaError_t e = cudaStreamQuery(c->stream);
    if (e == cudaSuccess) return 0;
    if (e != cudaErrorNotReady) {
      set_err("%s: %s", what, cudaGetErrorString(e));
      return CN_COMM_ERR_CUDA;
    }
    ncclResult_t st = ncclSuccess;
    if (ncclCommGetAsyncError(c->comm, &st) == ncclSuccess && st != ncclSuccess && st != ncclInProgress) {
      set_err("%s: %s", what, ncclGetErrorString(st));
      return CN_COMM_ERR_NCCL;
    }
    if (std::chrono::duration_cast<std::chrono::milliseconds>(Clock::now() - t0).count() > timeout_ms) {
      set_err("%s: not complete within %d ms (a rank did not arrive)", what, timeout_ms);
      return CN_COMM_ERR_TIMEOUT;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(100));
  }
}

void abort_comm(cn_comm* c) {
  if (c->comm && !c->aborted) {
    ncclCommAbort(c->comm);
    c->aborted = true;
  }
}
}  // namespace

extern "C" {

const char* cn_comm_last_error(void) { return g_err; }

int cn_comm_nccl_version(int* version) {
  if (!version) return CN_COMM_ERR_ARG;
  ncclResult_t r = ncclGetVersion(version);
  if (r != ncclSuccess) {
    set_err("ncclGetVersion: %s", ncclGetErrorString(r));
    return CN_COMM_ERR_NCCL;
  }
  return 0;
}

int cn_comm_unique_id(void* id) {
  static_assert(sizeof(ncclUniqueId) == CN_COMM_ID_BYTES, "NCCL unique id size");
  if (!id) {
    set_err("cn_comm_unique_id: null buffer");
    return CN_COMM_ERR_ARG;
  }
  ncclUniqueId u;
  ncclResult_t r = ncclGetUniqueId(&u);
  if (r != ncclSuccess) {
    set_err("ncclGetUniqueId: %s", ncclGetErrorString(r));
    return CN_COMM_ERR_NCCL;
  }
  memcpy(id, &u, sizeof(u));
  return 0;
}

int cn_comm_init(cn_comm** out, int device, int nranks, int rank, const void* id, int timeout_ms) {
  if (!out || !id || nranks < 1 || rank < 0 || rank >= nranks || timeout_ms <= 0) {
    set_err("cn_comm_init: bad arguments (nranks=%d rank=%d timeout_ms=%d)", nranks, rank, timeout_ms);
    return CN_COMM_ERR_ARG;
  }
  *out = nullptr;
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) {
    set_err("cn_comm_init: cudaSetDevice(%d): %s", device, cudaGetErrorString(e));
    return CN_COMM_ERR_CUDA;
  }
  cn_comm* c = new cn_comm();
  c->device = device;
  c->nranks = nranks;
  c->rank = rank;
  e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    set_err("cn_comm_init: stream: %s", cudaGetErrorString(e));
    delete c;
    return CN_COMM_ERR_CUDA;
  }
  ncclUniqueId u;
  memcpy(&u, id, sizeof(u));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclResult_t r = ncclCommInitRankConfig(&c->comm, nranks, u, rank, &cfg);
  int rc = 0;
  if (r != ncclSuccess && r != ncclInProgress) {
    set_err("ncclCommInitRankConfig: %s", ncclGetErrorString(r));
    rc = CN_COMM_ERR_NCCL;
  } else {
    rc = wait_comm(c, timeout_ms, "ncclCommInitRankConfig");
  }
  if (rc) {
    abort_comm(c);
    cudaStreamDestroy(c->stream);
    delete c;
    return rc;
  }
  *out = c;
  return 0;
}

int cn_comm_allgather_f64(cn_comm* c, const double* send, double* recv, size_t count, int timeout_ms) {
  if (!c || !send || !recv || count == 0 || timeout_ms <= 0) {
    set_err("cn_comm_allgather_f64: bad arguments");
    return CN_COMM_ERR_ARG;
  }
  if (c->aborted) {
    set_err("cn_comm_allgather_f64: the communicator was aborted by an earlier error");
    return CN_COMM_ERR_NCCL;
  }
  cudaError_t e = cudaSetDevice(c->device);
  if (e == cudaSuccess && count > c->cap) {
    if (c->dbuf) cudaFree(c->dbuf);
    c->dbuf = nullptr;
    c->cap = 0;
    e = cudaMalloc(&c->dbuf, (size_t)(c->nranks + 1) * count * sizeof(double));
    if (e == cudaSuccess) c->cap = count;
  }
  if (e != cudaSuccess) {
    set_err("cn_comm_allgather_f64: %s", cudaGetErrorString(e));
    return CN_COMM_ERR_CUDA;
  }
  double* dsend = c->dbuf + (size_t)c->nranks * count;
  e = cudaMemcpyAsync(dsend, send, count * sizeof(double), cudaMemcpyHostToDevice, c->stream);
  if (e != cudaSuccess) {
    set_err("cn_comm_allgather_f64: H2D: %s", cudaGetErrorString(e));
    return CN_COMM_ERR_CUDA;
  }
  ncclResult_t r = ncclAllGather(dsend, c->dbuf, count, ncclFloat64, c->comm, c->stream);
  int rc = 0;
  if (r != ncclSuccess && r != ncclInProgress) {
    set_err("ncclAllGather: %s", ncclGetErrorString(r));
    rc = CN_COMM_ERR_NCCL;
  } else if (r == ncclInProgress) {
    rc = wait_comm(c, timeout_ms, "ncclAllGather (enqueue)");
  }
  if (!rc) {
    e = cudaMemcpyAsync(recv, c->dbuf, (size_t)c->nranks * count * sizeof(double), cudaMemcpyDeviceToHost,
                        c->stream);
    if (e != cudaSuccess) {
      set_err("cn_comm_allgather_f64: D2H: %s", cudaGetErrorString(e));
      rc = CN_COMM_ERR_CUDA;
    }
  }
  if (!rc) rc = wait_stream(c, timeout_ms, "cn_comm_allgather_f64");
  if (rc == CN_COMM_ERR_TIMEOUT || rc == CN_COMM_ERR_NCCL) abort_comm(c);
  return rc;
}

int cn_comm_destroy(cn_comm* c) {
  if (!c) return 0;
  cudaSetDevice(c->device);
  if (c->comm) {
    if (!c->aborted) {
      // finalize flushes outstanding work; in non-blocking mode it may return in progress
      ncclResult_t r = ncclCommFinalize(c->comm);
      if (r == ncclSuccess || r == ncclInProgress) {
        if (wait_comm(c, 10000, "ncclCommFinalize")) {
          abort_comm(c);
        }
      } else {
        abort_comm(c);
      }
      if (!c->aborted) ncclCommDestroy(c->comm);
    }
  }
  if (c->dbuf) cudaFree(c->dbuf);
  if (c->stream) cudaStreamDestroy(c->stream);
  delete c;
  return 0;
}

}  // extern "C"
