// ep.cu — expert parallelism across GPUs: NCCL (loaded at run time) and the
// exchange plan of one MoE layer.
//
// With R ranks each GPU holds E / R consecutive experts of every layer (rank
// r: experts [r E_l, (r + 1) E_l)).  The router and the expert-major
// permutation of a rank's own tokens are unchanged: because a destination's
// experts are consecutive, the permuted operand is already grouped by
// destination rank, then by expert, then by token.  Per layer:
//   1. every rank sends each peer the counts of its routes to that peer's
//      experts (E_l ints), and receives the same from every source;
//   2. the plan (ep_plan below): rows to send to / receive from each peer,
//      and the local grouped-GEMM tiles over the received rows, which lie
//      source-major, then expert-major, then in the sources' token order;
//   3. the routed rows go out and come in (grouped ncclSend / ncclRecv), the
//      local experts run on the received rows, and their outputs go back to
//      the positions the rows had in the source's permuted operand -- the
//      layout the combine already reads, so the combine (ascending global
//      expert id per token, the reference's order, expert.ts:137-145) is the
//      single-GPU one.
// NCCL is not linked: libnccl.so.2 is opened when a handle enables expert
// parallelism (the copy already loaded by the process, if any), so the
// library has no NCCL dependency otherwise.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "ts_common.cuh"
#include "ts_ep.h"

namespace ts {
namespace {

struct NcclApi {
  bool ok = false;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

std::mutex g_nccl_mu;
NcclApi g_nccl;

template <typename F>
bool sym(void* lib, const char* name, F& f) {
  f = reinterpret_cast<F>(dlsym(lib, name));
  return f != nullptr;
}

const NcclApi* nccl(std::string* err) {
  std::lock_guard<std::mutex> lk(g_nccl_mu);
  if (g_nccl.ok) return &g_nccl;
  void* lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!lib) {
    if (err) *err = std::string("cannot open libnccl.so.2: ") + dlerror();
    return nullptr;
  }
  NcclApi a;
  if (!sym(lib, "ncclGetUniqueId", a.GetUniqueId) || !sym(lib, "ncclCommInitRank", a.CommInitRank) ||
      !sym(lib, "ncclCommDestroy", a.CommDestroy) || !sym(lib, "ncclCommAbort", a.CommAbort) ||
      !sym(lib, "ncclSend", a.Send) || !sym(lib, "ncclRecv", a.Recv) || !sym(lib, "ncclGroupStart", a.GroupStart) ||
      !sym(lib, "ncclGroupEnd", a.GroupEnd) || !sym(lib, "ncclGetErrorString", a.GetErrorString)) {
    if (err) *err = "libnccl.so.2 lacks an expected symbol";
    return nullptr;
  }
  a.ok = true;
  g_nccl = a;
  return &g_nccl;
}

std::string nccl_msg(const NcclApi* n, ncclResult_t r, const char* what) {
  return std::string(what) + ": " + (n ? n->GetErrorString(r) : "NCCL unavailable");
}

}  // namespace

bool ep_unique_id(void* out, size_t cap, std::string* err) {
  const NcclApi* n = nccl(err);
  if (!n) return false;
  if (cap < sizeof(ncclUniqueId)) {
    *err = "the id buffer needs " + std::to_string(sizeof(ncclUniqueId)) + " bytes";
    return false;
  }
  ncclUniqueId id;
  const ncclResult_t r = n->GetUniqueId(&id);
  if (r != ncclSuccess) {
    *err = nccl_msg(n, r, "ncclGetUniqueId");
    return false;
  }
  std::memcpy(out, &id, sizeof id);
  return true;
}

size_t ep_unique_id_bytes() { return sizeof(ncclUniqueId); }

bool ep_comm_init(void** comm, int world, const void* id, size_t id_len, int rank, std::string* err) {
  const NcclApi* n = nccl(err);
  if (!n) return false;
  if (id_len != sizeof(ncclUniqueId)) {
    *err = "the NCCL id must be " + std::to_string(sizeof(ncclUniqueId)) + " bytes";
    return false;
  }
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof uid);
  ncclComm_t c = nullptr;
  const ncclResult_t r = n->CommInitRank(&c, world, uid, rank);
  if (r != ncclSuccess) {
    *err = nccl_msg(n, r, "ncclCommInitRank");
    return false;
  }
  *comm = c;
  return true;
}

void ep_comm_destroy(void* comm, bool abort) {
  if (!comm) return;
  const NcclApi* n = nccl(nullptr);
  if (!n) return;
  if (abort) n->CommAbort(static_cast<ncclComm_t>(comm));
  else n->CommDestroy(static_cast<ncclComm_t>(comm));
}

bool ep_exchange(void* comm, int world, const void* send, const uint64_t* send_off, const uint64_t* send_n, void* recv,
                 const uint64_t* recv_off, const uint64_t* recv_n, size_t elem_bytes, cudaStream_t st,
                 std::string* err) {
  const NcclApi* n = nccl(err);
  if (!n) return false;
  // byte counts: every payload here is a whole number of 4-byte words
  const ncclDataType_t dt = elem_bytes % 4 == 0 ? ncclInt32 : ncclUint8;
  const size_t unit = elem_bytes % 4 == 0 ? 4 : 1;
  ncclComm_t c = static_cast<ncclComm_t>(comm);
  ncclResult_t r = n->GroupStart();
  for (int p = 0; p < world && r == ncclSuccess; p++) {
    if (send_n[p])
      r = n->Send(static_cast<const uint8_t*>(send) + send_off[p] * elem_bytes, send_n[p] * elem_bytes / unit, dt, p, c,
                  st);
    if (r == ncclSuccess && recv_n[p])
      r = n->Recv(static_cast<uint8_t*>(recv) + recv_off[p] * elem_bytes, recv_n[p] * elem_bytes / unit, dt, p, c, st);
  }
  const ncclResult_t r2 = n->GroupEnd();
  if (r != ncclSuccess || r2 != ncclSuccess) {
    *err = nccl_msg(n, r != ncclSuccess ? r : r2, "grouped ncclSend/ncclRecv");
    return false;
  }
  return true;
}

void ep_plan(const int* counts, const int* recv_counts, int world, int rank, int e_local, int tile_rows, EpPlan* out) {
  (void)rank;
  out->send_n.assign(world, 0);
  out->send_off.assign(world, 0);
  out->recv_n.assign(world, 0);
  out->recv_off.assign(world, 0);
  out->tiles.clear();
  uint64_t so = 0, ro = 0;
  for (int p = 0; p < world; p++) {
    uint64_t s = 0, r = 0;
    for (int j = 0; j < e_local; j++) {
      s += (uint64_t)counts[p * e_local + j];
      r += (uint64_t)recv_counts[p * e_local + j];
    }
    out->send_off[p] = so;
    out->send_n[p] = s;
    out->recv_off[p] = ro;
    out->recv_n[p] = r;
    so += s;
    ro += r;
  }
  out->send_total = so;
  out->recv_total = ro;
  // tiles: per local expert, the segment each source sent for it
  for (int j = 0; j < e_local; j++) {
    for (int p = 0; p < world; p++) {
      uint64_t seg = out->recv_off[p];
      for (int jj = 0; jj < j; jj++) seg += (uint64_t)recv_counts[p * e_local + jj];
      const uint64_t len = (uint64_t)recv_counts[p * e_local + j];
      for (uint64_t r0 = 0; r0 < len; r0 += (uint64_t)tile_rows) {
        const uint64_t r1 = std::min<uint64_t>(len, r0 + (uint64_t)tile_rows);
        out->tiles.push_back(make_int4(j, (int)(seg + r0), (int)(seg + r1), (int)seg));
      }
    }
  }
}

}  // namespace ts
