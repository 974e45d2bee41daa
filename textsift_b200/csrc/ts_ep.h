// ts_ep.h — expert parallelism across GPUs (ep.cu): NCCL loaded at run time
// and the exchange plan of one MoE layer.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace ts {

// The NCCL unique id (rank 0 makes it, every rank passes the same bytes).
size_t ep_unique_id_bytes();
bool ep_unique_id(void* out, size_t cap, std::string* err);
bool ep_comm_init(void** comm, int world, const void* id, size_t id_len, int rank, std::string* err);
void ep_comm_destroy(void* comm, bool abort);

// One grouped exchange: to peer p, send_n[p] elements of elem_bytes from
// send + send_off[p] elements; from peer p, recv_n[p] elements into recv +
// recv_off[p] elements (self included), enqueued on st.
bool ep_exchange(void* comm, int world, const void* send, const uint64_t* send_off, const uint64_t* send_n, void* recv,
                 const uint64_t* recv_off, const uint64_t* recv_n, size_t elem_bytes, cudaStream_t st,
                 std::string* err);

// The plan of one layer on one rank.  counts: this rank's routes per global
// expert [world * e_local] (expert-major = destination-major); recv_counts:
// routes each source sends to each local expert [world][e_local].  Send
// segments are consecutive in the permuted operand; received rows lie
// source-major, then local-expert-major; tiles = {local expert, first row,
// end row, segment start} of at most tile_rows rows over the received rows.
struct EpPlan {
  std::vector<uint64_t> send_n, send_off, recv_n, recv_off;
  uint64_t send_total = 0, recv_total = 0;
  std::vector<int4> tiles;
};
void ep_plan(const int* counts, const int* recv_counts, int world, int rank, int e_local, int tile_rows, EpPlan* out);

}  // namespace ts
