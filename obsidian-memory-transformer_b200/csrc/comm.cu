// comm.cu -- tensor-parallel communicator of the block (NCCL over NVLink /
// NVSwitch), loaded at run time.
//
// The library does not link NCCL: the first use opens libnccl.so.2 (the copy a
// host framework already loaded, e.g. PyTorch's, else the system one) and
// resolves the few entry points the block needs.  A communicator is created
// from a 128-byte unique id that rank 0 makes and the caller distributes over
// its own channel (torch.distributed, MPI, a file ...); every collective runs
// on the caller's stream, in stream order with the block's kernels.
#include <dlfcn.h>

#include <cstring>
#include <mutex>

#include <nccl.h>

#include "block.cuh"

namespace ltm_b200 {
namespace {

// Inside ncclGroupStart / End the collectives launch at the End: the kernel
// timer marks the group once there.
thread_local int t_group_depth = 0;

void note_collective(const char* what, cudaStream_t st) {
  if (t_group_depth == 0) note_launch(what, st);
}

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*reduce_scatter)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t,
                                 ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, int, ncclComm_t,
                         cudaStream_t) = nullptr;
  ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*group_start)() = nullptr;
  ncclResult_t (*group_end)() = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  ncclResult_t (*get_version)(int*) = nullptr;
  bool ok = false;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
    api.reduce_scatter =
        reinterpret_cast<decltype(api.reduce_scatter)>(dlsym(h, "ncclReduceScatter"));
    api.broadcast = reinterpret_cast<decltype(api.broadcast)>(dlsym(h, "ncclBroadcast"));
    api.reduce = reinterpret_cast<decltype(api.reduce)>(dlsym(h, "ncclReduce"));
    api.send = reinterpret_cast<decltype(api.send)>(dlsym(h, "ncclSend"));
    api.recv = reinterpret_cast<decltype(api.recv)>(dlsym(h, "ncclRecv"));
    api.group_start = reinterpret_cast<decltype(api.group_start)>(dlsym(h, "ncclGroupStart"));
    api.group_end = reinterpret_cast<decltype(api.group_end)>(dlsym(h, "ncclGroupEnd"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
    api.get_version = reinterpret_cast<decltype(api.get_version)>(dlsym(h, "ncclGetVersion"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_reduce &&
             api.all_gather && api.reduce_scatter && api.broadcast && api.reduce &&
             api.send && api.recv && api.group_start && api.group_end &&
             api.error_string;
  });
  if (!api.ok) {
    set_error("NCCL (libnccl.so.2) could not be loaded");
    throw Fail{LTM_ERR_COMM};
  }
  return api;
}

void nccl_check(ncclResult_t r, const char* what) {
  if (r != ncclSuccess) {
    set_error(std::string(what) + ": " + nccl().error_string(r));
    throw Fail{LTM_ERR_COMM};
  }
}

ncclDataType_t nccl_type(ltm_dtype dt) {
  switch (dt) {
    case LTM_DTYPE_F32: return ncclFloat32;
    case LTM_DTYPE_F16: return ncclFloat16;
    case LTM_DTYPE_BF16: return ncclBfloat16;
  }
  LTM_REQUIRE(false, "unknown dtype");
  return ncclFloat32;
}

}  // namespace

void comm_allreduce(ltm_comm* c, const void* send, void* recv, size_t count, ltm_dtype dt,
                    bool max_op, cudaStream_t st) {
  LTM_REQUIRE(c != nullptr, "NULL communicator");
  if (count == 0) return;
  nccl_check(nccl().all_reduce(send, recv, count, nccl_type(dt), max_op ? ncclMax : ncclSum,
                               static_cast<ncclComm_t>(c->handle), st),
             "ncclAllReduce");
  note_collective(max_op ? "nccl_allreduce/max" : "nccl_allreduce/sum", st);
}

void comm_allgather_bytes(ltm_comm* c, const void* send, void* recv, size_t bytes_per_rank,
                          cudaStream_t st) {
  LTM_REQUIRE(c != nullptr, "NULL communicator");
  if (bytes_per_rank == 0) return;
  nccl_check(nccl().all_gather(send, recv, bytes_per_rank, ncclInt8,
                               static_cast<ncclComm_t>(c->handle), st),
             "ncclAllGather");
  note_collective("nccl_allgather", st);
}

void comm_reduce_scatter(ltm_comm* c, const void* send, void* recv, size_t count_per_rank,
                         ltm_dtype dt, cudaStream_t st) {
  LTM_REQUIRE(c != nullptr, "NULL communicator");
  if (count_per_rank == 0) return;
  nccl_check(nccl().reduce_scatter(send, recv, count_per_rank, nccl_type(dt), ncclSum,
                                   static_cast<ncclComm_t>(c->handle), st),
             "ncclReduceScatter");
  note_collective("nccl_reduce_scatter", st);
}

void comm_broadcast_bytes(ltm_comm* c, void* buf, size_t bytes, int root, cudaStream_t st) {
  LTM_REQUIRE(c != nullptr, "NULL communicator");
  if (bytes == 0) return;
  nccl_check(nccl().broadcast(buf, buf, bytes, ncclInt8, root, static_cast<ncclComm_t>(c->handle),
                              st),
             "ncclBroadcast");
  note_collective("nccl_broadcast", st);
}

void comm_reduce(ltm_comm* c, const void* send, void* recv, size_t count, ltm_dtype dt, int root,
                 cudaStream_t st) {
  LTM_REQUIRE(c != nullptr, "NULL communicator");
  if (count == 0) return;
  nccl_check(nccl().reduce(send, recv, count, nccl_type(dt), ncclSum, root,
                           static_cast<ncclComm_t>(c->handle), st),
             "ncclReduce");
  note_collective("nccl_reduce", st);
}

void comm_send_recv_slots(ltm_comm* c, const void* send, void* recv, size_t bytes, int root,
                          cudaStream_t st) {
  LTM_REQUIRE(c != nullptr, "NULL communicator");
  if (bytes == 0) return;
  const ncclComm_t h = static_cast<ncclComm_t>(c->handle);
  comm_group_start();
  for (int j = 0; j < c->nranks; ++j) {
    if (j == c->rank) continue;
    if (root < 0 || root == j)  // this rank's rows of j's block go to j
      nccl_check(nccl().send(static_cast<const char*>(send) + j * bytes, bytes, ncclInt8, j, h, st),
                 "ncclSend");
    if (root < 0 || root == c->rank)  // j's partial of this rank's rows into slot j
      nccl_check(nccl().recv(static_cast<char*>(recv) + j * bytes, bytes, ncclInt8, j, h, st),
                 "ncclRecv");
  }
  comm_group_end(nullptr, st);
  note_collective("nccl_send_recv", st);
}

void comm_group_start() {
  nccl_check(nccl().group_start(), "ncclGroupStart");
  ++t_group_depth;
}

void comm_group_end(const char* what, cudaStream_t st) {
  --t_group_depth;
  nccl_check(nccl().group_end(), "ncclGroupEnd");
  if (what) note_collective(what, st);
}

}  // namespace ltm_b200

using namespace ltm_b200;

extern "C" ltm_status ltm_comm_unique_id(void* id_out) {
  return guarded([&] {
    LTM_REQUIRE(id_out != nullptr, "NULL id buffer");
    ncclUniqueId id;
    nccl_check(nccl().get_unique_id(&id), "ncclGetUniqueId");
    std::memcpy(id_out, &id, sizeof(id));
  });
}

extern "C" ltm_status ltm_comm_create(const void* id, int nranks, int rank, int device,
                                      ltm_comm** out) {
  return guarded([&] {
    LTM_REQUIRE(id && out, "NULL argument");
    LTM_REQUIRE(nranks >= 1 && rank >= 0 && rank < nranks, "rank outside [0, nranks)");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
      set_error("no CUDA device");
      throw Fail{LTM_ERR_NO_DEVICE};
    }
    LTM_REQUIRE(device >= 0 && device < ndev, "device index out of range");
    int prev = 0;
    LTM_CUDA_TRY(cudaGetDevice(&prev));
    LTM_CUDA_TRY(cudaSetDevice(device));
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    ncclComm_t comm = nullptr;
    const ncclResult_t r = nccl().comm_init_rank(&comm, nranks, uid, rank);
    cudaSetDevice(prev);
    nccl_check(r, "ncclCommInitRank");
    auto* c = new ltm_comm;
    c->handle = comm;
    c->nranks = nranks;
    c->rank = rank;
    c->device = device;
    *out = c;
  });
}

extern "C" ltm_status ltm_comm_allreduce(ltm_comm* comm, const void* send, void* recv,
                                         size_t count, ltm_dtype dtype, int op_max, void* stream) {
  return guarded([&] {
    LTM_REQUIRE(send && recv, "NULL buffer");
    comm_allreduce(comm, send, recv, count, dtype, op_max != 0, as_stream(stream));
  });
}

extern "C" ltm_status ltm_comm_destroy(ltm_comm* comm) {
  return guarded([&] {
    if (!comm) return;
    if (comm->handle) nccl_check(nccl().comm_destroy(static_cast<ncclComm_t>(comm->handle)),
                                 "ncclCommDestroy");
    delete comm;
  });
}
