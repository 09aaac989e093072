// Sequence-parallel (Ulysses) state of a handle; see sp.cu.
#pragma once
#include <cstddef>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace hx {

struct SpState {
  void* comm = nullptr;  // ncclComm_t
  int nranks = 1, rank = 0;
  void *send = nullptr, *recv = nullptr, *ofull = nullptr, *orecv = nullptr;  // exchange buffers
  size_t cap = 0;  // halves per q|k|v slice the buffers were sized for (Tl * D)
};

int sp_unique_id(void* out128);
int sp_comm_init(SpState& sp, int nranks, int rank, const void* id128);
void sp_comm_destroy(SpState& sp);
int sp_reserve(SpState& sp, size_t Tl, size_t D);
// ev: NULL, or 4 events recorded before the pack, after the q|k|v exchange, after the attention and after
// the o exchange + unpack (per-part timing of the block's attention stage)
cudaError_t sp_attention(SpState& sp, const __half* qkv, __half* O, int ldo, int Tl, int D, int H, int nvalid,
                         int* status, cudaStream_t s, cudaEvent_t* ev = nullptr);

}  // namespace hx
