// dist.cu -- NCCL communicator behind the reference's distributed backend
// (src/distributed/gpu_backend.cpp:66-130, abstract_backend.hpp:13-27).
//
// Differences from the reference: no MPI.  The 128-byte ncclUniqueId is
// produced on rank 0 and handed to the other ranks by the caller (a file,
// a TCP store, torch.distributed, ...); zl_comm_create_from_file() does it
// through a shared file with a bounded wait.  Communicator creation is
// non-blocking with a host deadline, and every collective can be checked
// with zl_comm_check(), which aborts the communicator if NCCL reports an
// asynchronous error or a deadline passes -- a rank that died makes the
// others fail with ZL_ETIMEOUT / ZL_ENCCL instead of hanging.
#include <nccl.h>
#include <unistd.h>

#include <chrono>
#include <cstdio>
#include <cstring>
#include <string>
#include <thread>

#include "common.cuh"

struct zl_comm {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1;
};

namespace {
bool to_nccl_type(int dtype, ncclDataType_t* t) {  // dist_types.hpp:19-25 order
  switch (dtype) {
    case 0: *t = ncclFloat32; return true;
    case 1: *t = ncclFloat16; return true;
    case 2: *t = ncclBfloat16; return true;
    case 3: *t = ncclInt32; return true;
    case 4: *t = ncclInt64; return true;
  }
  return false;
}
bool to_nccl_op(int op, ncclRedOp_t* o) {  // dist_types.hpp:10-16 order
  switch (op) {
    case 0: *o = ncclSum; return true;
    case 1: *o = ncclProd; return true;
    case 2: *o = ncclMin; return true;
    case 3: *o = ncclMax; return true;
    case 4: *o = ncclAvg; return true;
  }
  return false;
}
zl_status nccl_err(ncclResult_t r, const char* what) {
  return zl::set_error(ZL_ENCCL, "%s: %s", what, ncclGetErrorString(r));
}
// Polls a non-blocking communicator until `pred` holds or the deadline passes (then aborts it).
zl_status wait_ready(ncclComm_t comm, double timeout_s, const char* what) {
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    ncclResult_t st = ncclSuccess;
    ncclResult_t r = ncclCommGetAsyncError(comm, &st);
    if (r != ncclSuccess) return nccl_err(r, what);
    if (st == ncclSuccess) return ZL_OK;
    if (st != ncclInProgress) {
      ncclCommAbort(comm);
      return nccl_err(st, what);
    }
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > timeout_s) {
      ncclCommAbort(comm);
      return zl::set_error(ZL_ETIMEOUT, "%s: timed out after %.1f s", what, timeout_s);
    }
    std::this_thread::sleep_for(std::chrono::milliseconds(1));
  }
}
}  // namespace

extern "C" zl_status zl_comm_create(const void* id, int rank, int world, double timeout_s, zl_comm** out) {
  if (!id || !out || world <= 0 || rank < 0 || rank >= world) return zl::set_error(ZL_EINVAL, "comm_create: arguments");
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  zl_comm* c = new zl_comm();
  ncclResult_t r = ncclCommInitRankConfig(&c->comm, world, uid, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    delete c;
    return nccl_err(r, "ncclCommInitRankConfig");
  }
  zl_status s = wait_ready(c->comm, timeout_s, "ncclCommInitRankConfig");
  if (s != ZL_OK) {
    delete c;
    return s;
  }
  c->rank = rank;
  c->world = world;
  *out = c;
  return ZL_OK;
}

// Rank 0 creates the id and publishes it at `path` (atomic rename); other ranks wait for it.
extern "C" zl_status zl_comm_create_from_file(const char* path, int rank, int world, double timeout_s, zl_comm** out) {
  if (!path) return zl::set_error(ZL_EINVAL, "comm_create_from_file: null path");
  unsigned char id[128];
  if (rank == 0) {
    zl_status s = zl_nccl_unique_id(id, sizeof(id));
    if (s != ZL_OK) return s;
    std::string tmp = std::string(path) + ".tmp";
    FILE* f = fopen(tmp.c_str(), "wb");
    if (!f || fwrite(id, 1, sizeof(id), f) != sizeof(id)) {
      if (f) fclose(f);
      return zl::set_error(ZL_EINVAL, "comm_create_from_file: cannot write %s", tmp.c_str());
    }
    fclose(f);
    if (rename(tmp.c_str(), path) != 0) return zl::set_error(ZL_EINVAL, "comm_create_from_file: rename failed");
  } else {
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
      FILE* f = fopen(path, "rb");
      if (f) {
        const size_t got = fread(id, 1, sizeof(id), f);
        fclose(f);
        if (got == sizeof(id)) break;
      }
      if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > timeout_s)
        return zl::set_error(ZL_ETIMEOUT, "comm_create_from_file: no id at %s after %.1f s", path, timeout_s);
      std::this_thread::sleep_for(std::chrono::milliseconds(5));
    }
  }
  return zl_comm_create(id, rank, world, timeout_s, out);
}

extern "C" zl_status zl_comm_destroy(zl_comm* c) {
  if (!c) return ZL_OK;
  if (c->comm) ncclCommDestroy(c->comm);
  delete c;
  return ZL_OK;
}

extern "C" zl_status zl_comm_all_reduce(zl_comm* c, void* buf, size_t count, int dtype, int op, zl_stream s) {
  ncclDataType_t t;
  ncclRedOp_t o;
  if (!c || !to_nccl_type(dtype, &t) || !to_nccl_op(op, &o)) return zl::set_error(ZL_EINVAL, "all_reduce: arguments");
  ncclResult_t r = ncclAllReduce(buf, buf, count, t, o, c->comm, (cudaStream_t)s);
  return (r == ncclSuccess || r == ncclInProgress) ? ZL_OK : nccl_err(r, "ncclAllReduce");
}
extern "C" zl_status zl_comm_broadcast(zl_comm* c, void* buf, size_t count, int dtype, int root, zl_stream s) {
  ncclDataType_t t;
  if (!c || !to_nccl_type(dtype, &t)) return zl::set_error(ZL_EINVAL, "broadcast: arguments");
  ncclResult_t r = ncclBroadcast(buf, buf, count, t, root, c->comm, (cudaStream_t)s);
  return (r == ncclSuccess || r == ncclInProgress) ? ZL_OK : nccl_err(r, "ncclBroadcast");
}
extern "C" zl_status zl_comm_all_gather(zl_comm* c, const void* send, void* recv, size_t count, int dtype, zl_stream s) {
  ncclDataType_t t;
  if (!c || !to_nccl_type(dtype, &t)) return zl::set_error(ZL_EINVAL, "all_gather: arguments");
  ncclResult_t r = ncclAllGather(send, recv, count, t, c->comm, (cudaStream_t)s);
  return (r == ncclSuccess || r == ncclInProgress) ? ZL_OK : nccl_err(r, "ncclAllGather");
}
// Waits (bounded) for the stream's queued collectives; aborts the communicator on error or timeout.
extern "C" zl_status zl_comm_check(zl_comm* c, zl_stream s, double timeout_s) {
  if (!c) return zl::set_error(ZL_EINVAL, "comm_check: null");
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    cudaError_t q = cudaStreamQuery((cudaStream_t)s);
    if (q == cudaSuccess) break;
    if (q != cudaErrorNotReady) return zl::set_error(ZL_ECUDA, "comm_check: %s", cudaGetErrorString(q));
    ncclResult_t st = ncclSuccess;
    ncclCommGetAsyncError(c->comm, &st);
    if (st != ncclSuccess && st != ncclInProgress) {
      ncclCommAbort(c->comm);
      c->comm = nullptr;
      return nccl_err(st, "collective");
    }
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > timeout_s) {
      ncclCommAbort(c->comm);
      c->comm = nullptr;
      return zl::set_error(ZL_ETIMEOUT, "collective did not complete within %.1f s (peer lost?)", timeout_s);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
  return ZL_OK;
}
extern "C" zl_status zl_comm_rank(zl_comm* c, int* rank, int* world) {
  if (!c) return zl::set_error(ZL_EINVAL, "comm_rank: null");
  if (rank) *rank = c->rank;
  if (world) *world = c->world;
  return ZL_OK;
}
