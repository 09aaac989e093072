// Ulysses sequence parallelism for the MOSS joint attention (new in this runtime; the reference runs
// one device and has no collective).
//
// P ranks each hold T/P consecutive tokens of one image. Around the attention of a block:
//   pack      q|k|v [T/P][3D] -> send [c][dst][T/P][D/P]   (head group dst = heads [dst*H/P, (dst+1)*H/P))
//   exchange  NCCL grouped send/recv: rank r receives from rank j into recv[c][j*T/P ..] -> [c][T][D/P]
//   attention full sequence T over the local H/P heads (keys >= nvalid masked)
//   exchange  o [T][D/P]: rows of token block j go back to rank j -> orecv[j][T/P][D/P]
//   unpack    orecv -> O [T/P][D] (head group j at columns j*D/P)
// NCCL is loaded with dlopen on first use (the process's libnccl.so.2: torch's when torch is loaded).
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "hx_internal.h"
#include "hx_sp.h"

namespace hx {

namespace {

struct NcclApi {
  bool ok = false;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
};

NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!lib) return;
    api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(dlsym(lib, "ncclGetUniqueId"));
    api.CommInitRank = reinterpret_cast<decltype(api.CommInitRank)>(dlsym(lib, "ncclCommInitRank"));
    api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(dlsym(lib, "ncclCommDestroy"));
    api.Send = reinterpret_cast<decltype(api.Send)>(dlsym(lib, "ncclSend"));
    api.Recv = reinterpret_cast<decltype(api.Recv)>(dlsym(lib, "ncclRecv"));
    api.GroupStart = reinterpret_cast<decltype(api.GroupStart)>(dlsym(lib, "ncclGroupStart"));
    api.GroupEnd = reinterpret_cast<decltype(api.GroupEnd)>(dlsym(lib, "ncclGroupEnd"));
    api.ok = api.GetUniqueId && api.CommInitRank && api.CommDestroy && api.Send && api.Recv && api.GroupStart &&
             api.GroupEnd;
  });
  return api;
}

// send[c][j][i][e] = qkv[i][c*D + j*Dl + e], e < Dl = D/P; 8 halves per thread
__global__ void sp_pack_kernel(const __half* __restrict__ qkv, __half* __restrict__ send, int Tl, int D, int P) {
  const int Dl = D / P, V = Dl / 8;
  const long total = 3L * P * Tl * V;
  const long idx = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int v = static_cast<int>(idx % V);
  const long r = idx / V;
  const int i = static_cast<int>(r % Tl);
  const int j = static_cast<int>((r / Tl) % P);
  const int c = static_cast<int>(r / (static_cast<long>(Tl) * P));
  const uint4* src = reinterpret_cast<const uint4*>(qkv + static_cast<size_t>(i) * 3 * D + c * D + j * Dl) + v;
  reinterpret_cast<uint4*>(send)[idx] = *src;
}

// O[i][j*Dl + e] = orecv[j][i][e]
__global__ void sp_unpack_kernel(const __half* __restrict__ orecv, __half* __restrict__ O, int Tl, int D, int P,
                                 int ldo) {
  const int Dl = D / P, V = Dl / 8;
  const long total = static_cast<long>(P) * Tl * V;
  const long idx = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int v = static_cast<int>(idx % V);
  const long r = idx / V;
  const int i = static_cast<int>(r % Tl);
  const int j = static_cast<int>(r / Tl);
  reinterpret_cast<uint4*>(O + static_cast<size_t>(i) * ldo + j * Dl)[v] = reinterpret_cast<const uint4*>(orecv)[idx];
}

}  // namespace

int sp_unique_id(void* out128) {
  NcclApi& n = nccl();
  if (!n.ok || !out128) return -1;
  ncclUniqueId id;
  if (n.GetUniqueId(&id) != ncclSuccess) return -2;
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
  std::memcpy(out128, &id, sizeof id);
  return 0;
}

int sp_comm_init(SpState& sp, int nranks, int rank, const void* id128) {
  NcclApi& n = nccl();
  if (!n.ok) return -1;
  ncclUniqueId id;
  std::memcpy(&id, id128, sizeof id);
  ncclComm_t comm = nullptr;
  if (n.CommInitRank(&comm, nranks, id, rank) != ncclSuccess) return -2;
  sp.comm = comm;
  sp.nranks = nranks;
  sp.rank = rank;
  return 0;
}

void sp_comm_destroy(SpState& sp) {
  if (sp.comm) nccl().CommDestroy(static_cast<ncclComm_t>(sp.comm));
  sp.comm = nullptr;
  for (void* p : {sp.send, sp.recv, sp.ofull, sp.orecv}) cudaFree(p);
  sp.send = sp.recv = sp.ofull = sp.orecv = nullptr;
  sp.cap = 0;
}

int sp_reserve(SpState& sp, size_t Tl, size_t D) {
  const size_t need = Tl * D;  // halves per q|k|v slice of one rank
  if (sp.cap >= need) return 0;
  for (void* p : {sp.send, sp.recv, sp.ofull, sp.orecv}) cudaFree(p);
  sp.send = sp.recv = sp.ofull = sp.orecv = nullptr;
  sp.cap = 0;
  if (cudaMalloc(&sp.send, 3 * need * 2) != cudaSuccess || cudaMalloc(&sp.recv, 3 * need * 2) != cudaSuccess ||
      cudaMalloc(&sp.ofull, need * 2) != cudaSuccess || cudaMalloc(&sp.orecv, need * 2) != cudaSuccess)
    return -1;
  sp.cap = need;
  return 0;
}

// the Ulysses attention of one block: qkv [Tl][3D] -> O [Tl][D] (row pitch ldo)
cudaError_t sp_attention(SpState& sp, const __half* qkv, __half* O, int ldo, int Tl, int D, int H, int nvalid,
                         int* status, cudaStream_t s, cudaEvent_t* ev) {
  NcclApi& n = nccl();
  const int P = sp.nranks;
  if (!n.ok || !sp.comm || P < 2 || H % P || D % (8 * P) || static_cast<size_t>(Tl) * D > sp.cap)
    return cudaErrorInvalidValue;
  const int Dl = D / P, T = Tl * P;
  const size_t chunk = static_cast<size_t>(Tl) * Dl;  // halves per (c, peer) block
  __half* send = static_cast<__half*>(sp.send);
  __half* recv = static_cast<__half*>(sp.recv);
  __half* ofull = static_cast<__half*>(sp.ofull);
  __half* orecv = static_cast<__half*>(sp.orecv);
  ncclComm_t comm = static_cast<ncclComm_t>(sp.comm);
  if (ev) cudaEventRecord(ev[0], s);
  {
    const long total = 3L * P * Tl * (Dl / 8);
    sp_pack_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, s>>>(qkv, send, Tl, D, P);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  // every Send / Recv result is checked; a failed enqueue still closes the group before returning
  if (n.GroupStart() != ncclSuccess) return cudaErrorUnknown;
  bool ok = true;
  for (int j = 0; j < P && ok; ++j)
    for (int c = 0; c < 3 && ok; ++c) {
      ok = n.Send(send + (static_cast<size_t>(c) * P + j) * chunk, chunk, ncclHalf, j, comm, s) == ncclSuccess &&
           n.Recv(recv + static_cast<size_t>(c) * P * chunk + static_cast<size_t>(j) * chunk, chunk, ncclHalf, j,
                  comm, s) == ncclSuccess;
    }
  if (n.GroupEnd() != ncclSuccess || !ok) return cudaErrorUnknown;
  if (ev) cudaEventRecord(ev[1], s);
  AttnArgs a;
  a.q = recv;
  a.ldq = Dl;
  a.k = recv + static_cast<size_t>(P) * chunk;
  a.ldk = Dl;
  a.v = recv + 2 * static_cast<size_t>(P) * chunk;
  a.ldv = Dl;
  a.o = ofull;
  a.ldo = Dl;
  a.B = 1;
  a.H = H / P;
  a.Tq = T;
  a.Tk = T;
  a.nvalid = nvalid;
  a.status = status;
  cudaError_t e = attn_launch(a, s);
  if (e != cudaSuccess) return e;
  if (ev) cudaEventRecord(ev[2], s);
  if (n.GroupStart() != ncclSuccess) return cudaErrorUnknown;
  for (int j = 0; j < P && ok; ++j)
    ok = n.Send(ofull + static_cast<size_t>(j) * chunk, chunk, ncclHalf, j, comm, s) == ncclSuccess &&
         n.Recv(orecv + static_cast<size_t>(j) * chunk, chunk, ncclHalf, j, comm, s) == ncclSuccess;
  if (n.GroupEnd() != ncclSuccess || !ok) return cudaErrorUnknown;
  const long total = static_cast<long>(P) * Tl * (Dl / 8);
  sp_unpack_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, s>>>(orecv, O, Tl, D, P, ldo);
  e = cudaGetLastError();
  if (e == cudaSuccess && ev) cudaEventRecord(ev[3], s);
  return e;
}

}  // namespace hx
