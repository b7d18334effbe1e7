// Communicator interface used by va_api.cu (implemented in va_comm.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <string>

namespace va {

struct Comm;

bool comm_unique_id(void* out128, std::string* err);
Comm* comm_init(const void* id128, int nranks, int rank, std::string* err);
void comm_destroy(Comm* c, bool abort);
int comm_rank(const Comm* c);
int comm_size(const Comm* c);
// In-place all-gather of two bf16 buffers laid out as nranks equal slices of
// count_per_rank elements; this rank's slice is already in place.
bool comm_allgather_inplace2(Comm* c, void* buf_a, void* buf_b, size_t count_per_rank,
                             cudaStream_t st, std::string* err);
// All-gather of `bytes` bytes per rank: recv (device) receives nranks slices in rank
// order; send (device) holds this rank's slice.
bool comm_allgather_bytes(Comm* c, const void* send, void* recv, size_t bytes, cudaStream_t st,
                          std::string* err);
// True when the communicator reports an asynchronous failure (message in *err).
bool comm_async_error(Comm* c, std::string* err);

}  // namespace va
