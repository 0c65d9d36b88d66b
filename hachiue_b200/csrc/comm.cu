// comm.cu - single-process multi-GPU collectives for hosts that cannot run
// one process per GPU.  The reference's host is one Node process driving one
// GPUDevice (src/engine.ts:320); a multi-GPU 'cuda' backend under Node has
// to drive every GPU from that process, so the all-gather that joins the
// per-rank outputs of the sharded path (hachiue_b200/dist.py does the same with
// torch.distributed, one process per GPU) runs here on one NCCL communicator
// per device made by ncclCommInitAll, in one ncclGroupStart / ncclGroupEnd.
//
// NCCL is opened at the first hcu_comm_create with dlopen("libnccl.so.2"), not
// linked: a process that already holds an NCCL (torch's, for instance) shares
// it, and a library user who never creates a communicator never loads one.
#include <dlfcn.h>
#include <nccl.h>

#include <string.h>

#include <mutex>

#include "context.h"

struct hcu_comm_s {
  int n = 0;       // ranks driven by this process (devices[0..n), comms[0..n))
  int nranks = 0;  // ranks of the whole communicator (n, or the job's size for hcu_comm_init_rank)
  int devices[HCU_COMM_MAX_DEVICES] = {};
  ncclComm_t comms[HCU_COMM_MAX_DEVICES] = {};
};

namespace {

using hcu::fail;

struct NcclApi {
  decltype(&ncclCommInitAll) init_all = nullptr;
  decltype(&ncclCommInitRank) init_rank = nullptr;
  decltype(&ncclCommInitRankConfig) init_rank_config = nullptr;
  decltype(&ncclGetUniqueId) unique_id = nullptr;
  decltype(&ncclCommDestroy) destroy = nullptr;
  decltype(&ncclAllGather) all_gather = nullptr;
  decltype(&ncclGroupStart) group_start = nullptr;
  decltype(&ncclGroupEnd) group_end = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
  bool ok = false;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!lib) return;
    api.init_all = reinterpret_cast<decltype(api.init_all)>(dlsym(lib, "ncclCommInitAll"));
    api.init_rank = reinterpret_cast<decltype(api.init_rank)>(dlsym(lib, "ncclCommInitRank"));
    api.init_rank_config = reinterpret_cast<decltype(api.init_rank_config)>(dlsym(lib, "ncclCommInitRankConfig"));
    api.unique_id = reinterpret_cast<decltype(api.unique_id)>(dlsym(lib, "ncclGetUniqueId"));
    api.destroy = reinterpret_cast<decltype(api.destroy)>(dlsym(lib, "ncclCommDestroy"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(lib, "ncclAllGather"));
    api.group_start = reinterpret_cast<decltype(api.group_start)>(dlsym(lib, "ncclGroupStart"));
    api.group_end = reinterpret_cast<decltype(api.group_end)>(dlsym(lib, "ncclGroupEnd"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(lib, "ncclGetErrorString"));
    api.ok = api.init_all && api.init_rank && api.init_rank_config && api.unique_id && api.destroy &&
             api.all_gather && api.group_start && api.group_end && api.error_string;
  });
  return api;
}

int check_nccl(ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return HCU_OK;
  return fail(HCU_ENCCL, "%s: %s", what, nccl().error_string(r));
}

}  // namespace

extern "C" int hcu_comm_create(int n, const int* devices, hcu_comm* comm) {
  if (!comm || !devices) return fail(HCU_EINVAL, "hcu_comm_create: null argument");
  *comm = nullptr;
  if (n < 1 || n > HCU_COMM_MAX_DEVICES) return fail(HCU_EINVAL, "hcu_comm_create: %d devices (1..%d)", n,
                                                     HCU_COMM_MAX_DEVICES);
  int count = 0;
  HCU_TRY(hcu::check_cuda(cudaGetDeviceCount(&count), "hcu_comm_create: cudaGetDeviceCount"));
  for (int i = 0; i < n; i++) {
    if (devices[i] < 0 || devices[i] >= count)
      return fail(HCU_EINVAL, "hcu_comm_create: device %d of %d", devices[i], count);
    for (int j = 0; j < i; j++)
      if (devices[j] == devices[i]) return fail(HCU_EINVAL, "hcu_comm_create: device %d listed twice", devices[i]);
  }
  const NcclApi& api = nccl();
  if (!api.ok) return fail(HCU_ENCCL, "hcu_comm_create: libnccl.so.2 could not be opened");
  hcu_comm c = new (std::nothrow) hcu_comm_s;
  if (!c) return fail(HCU_ENOMEM, "hcu_comm_create: out of host memory");
  c->n = n;
  c->nranks = n;
  for (int i = 0; i < n; i++) c->devices[i] = devices[i];
  const int st = check_nccl(api.init_all(c->comms, n, c->devices), "hcu_comm_create: ncclCommInitAll");
  if (st != HCU_OK) {
    delete c;
    return st;
  }
  *comm = c;
  return HCU_OK;
}

extern "C" int hcu_comm_unique_id(uint8_t* id) {
  if (!id) return fail(HCU_EINVAL, "hcu_comm_unique_id: null argument");
  static_assert(sizeof(ncclUniqueId) == HCU_COMM_ID_BYTES, "NCCL unique id size");
  const NcclApi& api = nccl();
  if (!api.ok) return fail(HCU_ENCCL, "hcu_comm_unique_id: libnccl.so.2 could not be opened");
  ncclUniqueId uid;
  HCU_TRY(check_nccl(api.unique_id(&uid), "hcu_comm_unique_id: ncclGetUniqueId"));
  memcpy(id, &uid, sizeof(uid));
  return HCU_OK;
}

extern "C" int hcu_comm_init_rank(int nranks, int rank, const uint8_t* id, int device, int max_ctas,
                                  hcu_comm* comm) {
  if (!comm || !id) return fail(HCU_EINVAL, "hcu_comm_init_rank: null argument");
  *comm = nullptr;
  if (nranks < 1 || rank < 0 || rank >= nranks)
    return fail(HCU_EINVAL, "hcu_comm_init_rank: rank %d of %d", rank, nranks);
  int count = 0;
  HCU_TRY(hcu::check_cuda(cudaGetDeviceCount(&count), "hcu_comm_init_rank: cudaGetDeviceCount"));
  if (device < 0 || device >= count) return fail(HCU_EINVAL, "hcu_comm_init_rank: device %d of %d", device, count);
  if (max_ctas < 0) return fail(HCU_EINVAL, "hcu_comm_init_rank: max_ctas %d", max_ctas);
  const NcclApi& api = nccl();
  if (!api.ok) return fail(HCU_ENCCL, "hcu_comm_init_rank: libnccl.so.2 could not be opened");
  HCU_TRY(hcu::check_cuda(cudaSetDevice(device), "hcu_comm_init_rank: cudaSetDevice"));
  hcu_comm c = new (std::nothrow) hcu_comm_s;
  if (!c) return fail(HCU_ENOMEM, "hcu_comm_init_rank: out of host memory");
  c->n = 1;
  c->nranks = nranks;
  c->devices[0] = device;
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  int st;
  if (max_ctas > 0) {
    // Collectives of this communicator occupy at most max_ctas SMs: the path's
    // per-step all-gathers are small and overlap the next step's kernels,
    // which need the SMs more than the gather needs channels.
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.minCTAs = 1;
    cfg.maxCTAs = max_ctas;
    st = check_nccl(api.init_rank_config(&c->comms[0], nranks, uid, rank, &cfg),
                    "hcu_comm_init_rank: ncclCommInitRankConfig");
  } else {
    st = check_nccl(api.init_rank(&c->comms[0], nranks, uid, rank), "hcu_comm_init_rank: ncclCommInitRank");
  }
  if (st != HCU_OK) {
    delete c;
    return st;
  }
  *comm = c;
  return HCU_OK;
}

extern "C" int hcu_comm_destroy(hcu_comm comm) {
  if (!comm) return HCU_OK;
  int st = HCU_OK;
  for (int i = 0; i < comm->n; i++) {
    const int r = check_nccl(nccl().destroy(comm->comms[i]), "hcu_comm_destroy: ncclCommDestroy");
    if (st == HCU_OK) st = r;
  }
  delete comm;
  return st;
}

extern "C" int hcu_allgather(hcu_comm comm, void* const* send, void* const* recv, size_t bytes,
                             void* const* streams) {
  if (!comm || !send || !recv || !streams) return fail(HCU_EINVAL, "hcu_allgather: null argument");
  for (int i = 0; i < comm->n; i++)
    if (!send[i] || !recv[i]) return fail(HCU_EINVAL, "hcu_allgather: null buffer of rank %d", i);
  if (bytes == 0) return HCU_OK;
  const NcclApi& api = nccl();
  int prev = 0;
  HCU_TRY(hcu::check_cuda(cudaGetDevice(&prev), "hcu_allgather: cudaGetDevice"));
  // Every check that can fail runs before ncclGroupStart: once the group is
  // open, a rank left out would make the others' all-gathers wait for it.
  for (int i = 0; i < comm->n; i++) {
    HCU_TRY(hcu::check_cuda(cudaSetDevice(comm->devices[i]), "hcu_allgather: cudaSetDevice"));
    if (streams[i]) {
      int sdev = -1;
      cudaStream_t s = static_cast<cudaStream_t>(streams[i]);
      int st = hcu::check_cuda(cudaStreamGetDevice(s, &sdev), "hcu_allgather: stream device");
      if (st == HCU_OK && sdev != comm->devices[i])
        st = fail(HCU_EINVAL, "hcu_allgather: stream of rank %d is on device %d, not %d", i, sdev, comm->devices[i]);
      if (st != HCU_OK) {
        cudaSetDevice(prev);
        return st;
      }
    }
  }
  HCU_TRY(check_nccl(api.group_start(), "hcu_allgather: ncclGroupStart"));
  // Inside the group only NCCL calls (whose errors NCCL itself knows about
  // and reports at ncclGroupEnd) and cudaSetDevice on devices checked above.
  ncclResult_t first = ncclSuccess;
  for (int i = 0; i < comm->n; i++) {
    cudaSetDevice(comm->devices[i]);
    const ncclResult_t r = api.all_gather(send[i], recv[i], bytes, ncclInt8, comm->comms[i],
                                          static_cast<cudaStream_t>(streams[i]));
    if (r != ncclSuccess && first == ncclSuccess) first = r;
  }
  const int end = check_nccl(api.group_end(), "hcu_allgather: ncclGroupEnd");
  cudaSetDevice(prev);
  if (first != ncclSuccess) return check_nccl(first, "hcu_allgather: ncclAllGather");
  return end;
}
