// Multi-GPU layer: one process per GPU, the hot path sharded into independent
// units (token rows of the GEMM, (batch, kv-head group) units of attention)
// and the outputs gathered over NVLink.  The reference names this exchange
// only as an IR collective (include/jules/Dialect/JulesOps.td:660-684) whose
// lowering is dead code; the partition follows its shapes.
//
// Plumbing: NCCL, loaded at run time (dlopen "libnccl.so.2": in a process that
// already holds one, e.g. PyTorch's, that library is reused), for the
// communicator, the exchange of peer-memory handles and the attention gather.
//
// Gather fused into the kernel: when the output is a "shared" buffer
// (cudaMalloc + CUDA IPC handles exchanged over the communicator), the GEMM
// (or attention) epilogue stores each finished tile of this rank's rows (or
// units) into every rank's output over NVLink while later tiles are still
// being computed.  A one-thread kernel then signals every rank (system-scope
// atomics on a counter in each rank's memory) and waits, with a bounded
// spin, until all ranks have signalled: after it, every rank's output holds
// the whole result.  Outputs that are not shared fall back to computing the
// local share and an in-place ncclAllGather.
//
// NVLink multicast: when the loaded NCCL has the symmetric-memory device API
// (NCCL 2.28, the version of the headers this file is compiled against) and
// the node's NVSwitch supports multicast (NVLS), shared buffers are NCCL
// symmetric windows (ncclMemAlloc + ncclCommWindowRegister) and the
// communicator carries a multicast handle (ncclDevCommCreate with
// lsaMultimem): the epilogues then store each 16-byte chunk once, to the
// buffer's multicast address, and the switch writes it into every rank's
// buffer.  Opt-in (JULES_DIST_MULTICAST=1); otherwise, and without that NCCL
// or NVLS, the buffers are cudaMalloc + CUDA IPC and the epilogues store to
// each rank.
#pragma once

#include <dlfcn.h>
#include <nccl.h>

#if __has_include(<nccl_device.h>)
#include <nccl_device.h>
#define JULES_NCCL_DEVICE_API 1
#else
#define JULES_NCCL_DEVICE_API 0
#endif

#include <cstdlib>
#include <vector>

namespace jb {
namespace dist {

constexpr int kMaxRanks = 8;  // == gemm::kMaxOutDest
constexpr uint32_t kSiteSignalWait = 251;

// Adds one to every rank's completion counter, then waits until this rank's
// counter reaches `target` (= world x calls so far).  One thread.  The
// fence before the signals orders this rank's earlier peer stores (the
// GEMM epilogue also fences them system-wide before its kernel ends).
__global__ void dist_signal_wait_kernel(unsigned long long* const* counters, int world,
                                        const unsigned long long* mine,
                                        unsigned long long target, uint64_t limit_ns) {
  if (threadIdx.x != 0) return;
  __threadfence_system();
  for (int r = 0; r < world; ++r) atomicAdd_system(counters[r], 1ull);
  const uint64_t t0 = globaltimer();
  for (uint32_t it = 1;; ++it) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(mine) : "memory");
    if (v >= target) break;
    if ((it & 63u) == 0 && globaltimer() - t0 > limit_ns) {
      record_error(kDevErrTimeout, kSiteSignalWait);
      return;
    }
    __nanosleep(64);
  }
  __threadfence_system();
}

#if JULES_NCCL_DEVICE_API
// A symmetric window's multicast address (out[0]) and every rank's unicast
// address of it (out[1 + r]), resolved by NCCL's own device functions.
__global__ void window_ptrs_kernel(ncclWindow_t w, ncclDevComm dc, int world, void** out) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  out[0] = ncclGetLsaMultimemPointer(w, 0, dc);
  for (int r = 0; r < world; ++r) out[1 + r] = ncclGetLsaPointer(w, 0, r);
}
#endif

}  // namespace dist
}  // namespace jb

namespace {

// ---------------------------------------------------------------------------
// NCCL entry points, resolved once.
// ---------------------------------------------------------------------------
struct NcclApi {
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRank) comm_init_rank = nullptr;
  decltype(&ncclCommDestroy) comm_destroy = nullptr;
  decltype(&ncclAllGather) all_gather = nullptr;
  decltype(&ncclAllReduce) all_reduce = nullptr;
  decltype(&ncclBroadcast) broadcast = nullptr;
  decltype(&ncclGroupStart) group_start = nullptr;
  decltype(&ncclGroupEnd) group_end = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
  decltype(&ncclGetVersion) get_version = nullptr;
#if JULES_NCCL_DEVICE_API
  // Symmetric windows and the device communicator (optional).
  decltype(&ncclMemAlloc) mem_alloc = nullptr;
  decltype(&ncclMemFree) mem_free = nullptr;
  decltype(&ncclCommWindowRegister) win_register = nullptr;
  decltype(&ncclCommWindowDeregister) win_deregister = nullptr;
  decltype(&ncclDevCommCreate) devcomm_create = nullptr;
  decltype(&ncclDevCommDestroy) devcomm_destroy = nullptr;
#endif
  bool device_api = false;  // all of those, from a library of the headers' version
  int version = 0;
  bool loaded = false;
  std::string why;
};

NcclApi& nccl_lib() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
    if (!h) {
      const char* e = dlerror();
      api.why = e ? e : "dlopen(libnccl.so.2) failed";
      return;
    }
    bool ok = true;
    auto sym = [&](auto& fn, const char* name) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
      if (!fn) ok = false;
    };
    sym(api.get_unique_id, "ncclGetUniqueId");
    sym(api.comm_init_rank, "ncclCommInitRank");
    sym(api.comm_destroy, "ncclCommDestroy");
    sym(api.all_gather, "ncclAllGather");
    sym(api.all_reduce, "ncclAllReduce");
    sym(api.broadcast, "ncclBroadcast");
    sym(api.group_start, "ncclGroupStart");
    sym(api.group_end, "ncclGroupEnd");
    sym(api.error_string, "ncclGetErrorString");
    api.loaded = ok;
    if (!ok) api.why = "libnccl.so.2 lacks an expected symbol";
    auto opt = [&](auto& fn, const char* name) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
      return fn != nullptr;
    };
    if (opt(api.get_version, "ncclGetVersion")) api.get_version(&api.version);
#if JULES_NCCL_DEVICE_API
    bool dev = opt(api.mem_alloc, "ncclMemAlloc");
    dev = opt(api.mem_free, "ncclMemFree") && dev;
    dev = opt(api.win_register, "ncclCommWindowRegister") && dev;
    dev = opt(api.win_deregister, "ncclCommWindowDeregister") && dev;
    dev = opt(api.devcomm_create, "ncclDevCommCreate") && dev;
    dev = opt(api.devcomm_destroy, "ncclDevCommDestroy") && dev;
    // The device communicator and window structs are read by code compiled
    // from this version's headers.
    api.device_api = ok && dev && api.version == NCCL_VERSION_CODE;
#endif
  });
  return api;
}

int nccl_fail(ncclResult_t r, const char* what) {
  return fail(JULES_ERR_COMM, "%s: %s", what, nccl_lib().error_string ? nccl_lib().error_string(r) : "?");
}

int need_nccl() {
  if (!nccl_lib().loaded) return fail(JULES_ERR_COMM, "NCCL unavailable: %s", nccl_lib().why.c_str());
  return JULES_OK;
}

// ---------------------------------------------------------------------------
// Communicator state.
// ---------------------------------------------------------------------------
struct SharedBuf {
  void* local = nullptr;
  size_t bytes = 0;
  void* peers[jb::dist::kMaxRanks] = {};  // peers[rank] == local
  void* mc = nullptr;   // multicast address of the whole buffer (symmetric window), or null
  void* win = nullptr;  // ncclWindow_t of a symmetric window, or null (cudaMalloc + IPC)
};

struct DistComm {
  ncclComm_t comm = nullptr;
  int world = 1, rank = 0, dev = 0;
  bool multicast = false;  // shared buffers are multicast windows, stored through their
                           // multicast address
#if JULES_NCCL_DEVICE_API
  bool has_devcomm = false;
  ncclDevComm devcomm{};
#endif
  unsigned long long calls = 0;             // signal/wait rounds issued (same on every rank)
  SharedBuf flags;                          // one u64 completion counter per rank
  unsigned long long** d_counters = nullptr;  // device array: every rank's counter
  std::vector<SharedBuf> shared;            // buffers from jules_dist_alloc_shared
  std::mutex mu;
  // Pull gather: one side stream per peer for its copy, fork / join events.
  cudaStream_t side[jb::dist::kMaxRanks] = {};
  cudaEvent_t fork = nullptr, join[jb::dist::kMaxRanks] = {};
  int gather_mode = 0;  // 0 auto, 1 fused stores, 2 pull (JULES_DIST_GATHER)
};

void side_release(DistComm* c) {
  for (int q = 0; q < jb::dist::kMaxRanks; ++q) {
    if (c->side[q]) cudaStreamDestroy(c->side[q]);
    if (c->join[q]) cudaEventDestroy(c->join[q]);
    c->side[q] = nullptr;
    c->join[q] = nullptr;
  }
  if (c->fork) cudaEventDestroy(c->fork);
  c->fork = nullptr;
}

// Whether a sharded call with a shared output of `out_bytes` gathers by
// pulling (copy engines, after the kernel) instead of by the epilogue's
// stores to every rank.  JULES_DIST_GATHER=stores / pull forces one; the
// same answer on every rank (world, sizes and the variable are).  Stores by
// default: on 8 B200s of one box (same run, back to back) the pull route
// measured C2 GEMM 732 vs 1215 TFLOP/s, C3 attention 982 vs 1815, C5 3266 vs
// 6535 - the copy engines brought ~260 GB/s into each GPU, the epilogue's
// stores overlap the kernel's own compute.
bool use_pull_gather(const DistComm* c, size_t out_bytes) {
  (void)out_bytes;
  return c->gather_mode == 2;
}

// Pull gather of a shared buffer whose rank shares are contiguous: after the
// signal/wait round (every rank's share is complete), copy each peer's share
// [begin_q, end_q) x unit_bytes from its buffer into ours, one copy engine
// transfer per peer on its own side stream, joined back into `st`.  The
// same for a second buffer (the attention lse) when buf2 is set.
int pull_gather(DistComm* c, const SharedBuf& buf, int64_t units, size_t unit_bytes,
                const SharedBuf* buf2, size_t unit_bytes2, cudaStream_t st) {
  cudaError_t e = cudaSuccess;
  if (!c->fork) {
    e = cudaEventCreateWithFlags(&c->fork, cudaEventDisableTiming);
    for (int q = 0; q < c->world && e == cudaSuccess; ++q) {
      e = cudaStreamCreateWithFlags(&c->side[q], cudaStreamNonBlocking);
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->join[q], cudaEventDisableTiming);
    }
    if (e != cudaSuccess) {
      side_release(c);
      return cuda_fail(e, "pull gather streams");
    }
  }
  if ((e = cudaEventRecord(c->fork, st)) != cudaSuccess) return cuda_fail(e, "pull gather fork");
  for (int q = 0; q < c->world; ++q) {
    if (q == c->rank) continue;
    int64_t b, en;
    jules_dist_shard(units, c->world, q, &b, &en);
    if (en <= b) continue;
    e = cudaStreamWaitEvent(c->side[q], c->fork, 0);
    const size_t off = (size_t)b * unit_bytes, n = (size_t)(en - b) * unit_bytes;
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(static_cast<char*>(buf.local) + off, static_cast<const char*>(buf.peers[q]) + off, n,
                          cudaMemcpyDeviceToDevice, c->side[q]);
    if (e == cudaSuccess && buf2) {
      const size_t off2 = (size_t)b * unit_bytes2, n2 = (size_t)(en - b) * unit_bytes2;
      e = cudaMemcpyAsync(static_cast<char*>(buf2->local) + off2,
                          static_cast<const char*>(buf2->peers[q]) + off2, n2, cudaMemcpyDeviceToDevice,
                          c->side[q]);
    }
    if (e == cudaSuccess) e = cudaEventRecord(c->join[q], c->side[q]);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(st, c->join[q], 0);
    if (e != cudaSuccess) return cuda_fail(e, "pull gather copy");
  }
  return JULES_OK;
}

// Collective for symmetric windows (the deregistration is), local for IPC
// buffers.
void shared_release(DistComm* c, SharedBuf& b) {
#if JULES_NCCL_DEVICE_API
  if (b.win) {
    nccl_lib().win_deregister(c->comm, static_cast<ncclWindow_t>(b.win));
    nccl_lib().mem_free(b.local);
    b = SharedBuf{};
    return;
  }
#endif
  for (int r = 0; r < c->world; ++r)
    if (r != c->rank && b.peers[r]) cudaIpcCloseMemHandle(b.peers[r]);
  if (b.local) cudaFree(b.local);
  b = SharedBuf{};
}

#if JULES_NCCL_DEVICE_API
// Collective: a symmetric window of `bytes` (rounded up to 4 KiB) on every
// rank, zeroed, with its multicast address and every rank's unicast address.
int shared_alloc_window(DistComm* c, size_t bytes, SharedBuf* out) {
  SharedBuf b;
  b.bytes = bytes;
  const size_t sz = (bytes + 4095) & ~size_t(4095);
  ncclResult_t r = nccl_lib().mem_alloc(&b.local, sz);
  if (r != ncclSuccess) return nccl_fail(r, "ncclMemAlloc");
  cudaError_t e = cudaMemset(b.local, 0, sz);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    nccl_lib().mem_free(b.local);
    return cuda_fail(e, "cudaMemset(shared window)");
  }
  ncclWindow_t w = nullptr;
  r = nccl_lib().win_register(c->comm, b.local, sz, &w, NCCL_WIN_COLL_SYMMETRIC);
  if (r != ncclSuccess) {
    nccl_lib().mem_free(b.local);
    return nccl_fail(r, "ncclCommWindowRegister");
  }
  b.win = w;
  void** d = nullptr;
  void* h[1 + jb::dist::kMaxRanks] = {};
  const size_t hb = sizeof(void*) * (1 + c->world);
  e = cudaMalloc(&d, hb);
  if (e == cudaSuccess) {
    jb::dist::window_ptrs_kernel<<<1, 32>>>(w, c->devcomm, c->world, d);
    e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaMemcpy(h, d, hb, cudaMemcpyDeviceToHost);
    cudaFree(d);
  }
  if (e != cudaSuccess || !h[0]) {
    shared_release(c, b);
    return e != cudaSuccess ? cuda_fail(e, "symmetric window addresses")
                            : fail(JULES_ERR_COMM, "symmetric window without a multicast address");
  }
  b.mc = h[0];
  for (int q = 0; q < c->world; ++q) b.peers[q] = q == c->rank ? b.local : h[1 + q];
  *out = b;
  return JULES_OK;
}

// Collective: the device communicator with a multicast handle, when every
// rank can have one and JULES_DIST_MULTICAST=1 asks for it.  c->multicast
// says whether shared buffers are windows and the fused gathers store
// through their multicast address.  Off by default: a multicast store also
// sends this rank's own share out through the switch and back (each GPU
// receives the whole output instead of (world-1)/world of it), and on 2, 4
// and 8 B200s of one NVSwitch node it measured no reproducible gain over
// peer stores (8 ranks: C2 GEMM 1200 and 1054 TFLOP/s on two boxes against
// 1075, C3 attention 2096 and 1741 against 1783; a long C5 attention 4062
// against 6467; 4 ranks: C2 1105 against 1466; 2 ranks: C2 1197 against
// 1499).
void multicast_setup(DistComm* c) {
  if (c->world < 2) return;
  const char* env = std::getenv("JULES_DIST_MULTICAST");
  int want = nccl_lib().device_api && env && env[0] == '1' ? 1 : 0;
  // Every rank must take the same allocation route: agree on the flag first.
  int* d = nullptr;
  if (cudaMalloc(&d, sizeof(int)) != cudaSuccess) return;
  int agreed = 0;
  if (cudaMemcpy(d, &want, sizeof(int), cudaMemcpyHostToDevice) == cudaSuccess &&
      nccl_lib().all_reduce(d, d, 1, ncclInt32, ncclMin, c->comm, nullptr) == ncclSuccess &&
      cudaMemcpy(&agreed, d, sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess && agreed) {
    ncclDevCommRequirements reqs{};
    reqs.lsaMultimem = true;
    int have = 0;
    if (nccl_lib().devcomm_create(c->comm, &reqs, &c->devcomm) == ncclSuccess) {
      c->has_devcomm = true;
      have = c->devcomm.lsaMultimem.mcBasePtr != nullptr && c->devcomm.lsaSize == c->world &&
             c->devcomm.lsaRank == c->rank;
    }
    int all = 0;
    if (cudaMemcpy(d, &have, sizeof(int), cudaMemcpyHostToDevice) == cudaSuccess &&
        nccl_lib().all_reduce(d, d, 1, ncclInt32, ncclMin, c->comm, nullptr) == ncclSuccess &&
        cudaMemcpy(&all, d, sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess)
      c->multicast = all != 0;
  }
  cudaFree(d);
}
#endif

// Collective: every rank allocates `bytes`, exports a CUDA IPC handle, the
// handles are all-gathered over NCCL and each rank maps the others'.
int shared_alloc(DistComm* c, size_t bytes, SharedBuf* out) {
  SharedBuf b;
  b.bytes = bytes;
  cudaError_t e = cudaMalloc(&b.local, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(shared buffer)");
  e = cudaMemset(b.local, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();  // zeroed before any peer can map it
  if (e != cudaSuccess) {
    cudaFree(b.local);
    return cuda_fail(e, "cudaMemset(shared buffer)");
  }
  cudaIpcMemHandle_t mine;
  e = cudaIpcGetMemHandle(&mine, b.local);
  const size_t hb = sizeof(cudaIpcMemHandle_t);
  char* d_handles = nullptr;
  if (e == cudaSuccess) e = cudaMalloc(&d_handles, hb * c->world);
  if (e != cudaSuccess) {
    cudaFree(b.local);
    return cuda_fail(e, "cudaIpcGetMemHandle / handle exchange buffer");
  }
  std::vector<cudaIpcMemHandle_t> all(c->world);
  int rc = JULES_OK;
  cudaStream_t st = nullptr;
  if ((e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking)) != cudaSuccess) {
    rc = cuda_fail(e, "cudaStreamCreate");
  } else if ((e = cudaMemcpy(d_handles + hb * c->rank, &mine, hb, cudaMemcpyHostToDevice)) != cudaSuccess) {
    rc = cuda_fail(e, "copy IPC handle");
  } else {
    ncclResult_t r = nccl_lib().all_gather(d_handles + hb * c->rank, d_handles, hb, ncclUint8, c->comm, st);
    if (r != ncclSuccess) rc = nccl_fail(r, "ncclAllGather(IPC handles)");
    else if ((e = cudaStreamSynchronize(st)) != cudaSuccess) rc = cuda_fail(e, "handle exchange");
    else if ((e = cudaMemcpy(all.data(), d_handles, hb * c->world, cudaMemcpyDeviceToHost)) != cudaSuccess)
      rc = cuda_fail(e, "copy IPC handles");
  }
  if (st) cudaStreamDestroy(st);
  cudaFree(d_handles);
  if (rc) {
    cudaFree(b.local);
    return rc;
  }
  for (int r = 0; r < c->world; ++r) {
    if (r == c->rank) {
      b.peers[r] = b.local;
      continue;
    }
    e = cudaIpcOpenMemHandle(&b.peers[r], all[r], cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      b.peers[r] = nullptr;
      shared_release(c, b);
      return cuda_fail(e, "cudaIpcOpenMemHandle");
    }
  }
  *out = b;
  return JULES_OK;
}

// The shared buffer starting at ptr with at least `bytes`, if any.
bool find_shared(DistComm* c, const void* ptr, size_t bytes, SharedBuf* out) {
  std::lock_guard<std::mutex> lk(c->mu);
  for (const auto& s : c->shared)
    if (s.local == ptr && s.bytes >= bytes) {
      *out = s;
      return true;
    }
  return false;
}

int dist_check(void* comm, DistComm** c) {
  if (!comm) return fail(JULES_ERR_ARG, "dist: NULL communicator");
  *c = static_cast<DistComm*>(comm);
  int dev;
  if (int rc = current_device(&dev)) return rc;
  if (dev != (*c)->dev) return fail(JULES_ERR_ARG, "dist: device %d is current, the communicator is on %d", dev, (*c)->dev);
  return JULES_OK;
}

int nccl_type(int dtype, ncclDataType_t* t) {
  switch (dtype) {
    case JULES_DTYPE_F32: *t = ncclFloat32; return JULES_OK;
    case JULES_DTYPE_BF16: *t = ncclBfloat16; return JULES_OK;
    case JULES_DTYPE_F16: *t = ncclFloat16; return JULES_OK;
    case JULES_DTYPE_FP8E4M3:
    case JULES_DTYPE_FP8E5M2: *t = ncclUint8; return JULES_OK;
    default: return fail(JULES_ERR_DTYPE, "dist: dtype %d", dtype);
  }
}

size_t dtype_bytes(int dtype) {
  return dtype == JULES_DTYPE_F32 ? 4 : ((dtype == JULES_DTYPE_BF16 || dtype == JULES_DTYPE_F16) ? 2 : 1);
}

// Gathers rank slices of `elems_total` elements (rank r owns [begin_r, end_r)
// of a balanced contiguous partition of `units` units of `unit_elems` each)
// in place: an ncclAllGather when the partition is equal, else one
// broadcast per rank in a group.
int gather_in_place(DistComm* c, void* buf, int64_t units, int64_t unit_elems, ncclDataType_t t,
                    size_t elt, cudaStream_t st) {
  const int w = c->world;
  char* base = static_cast<char*>(buf);
  if (units % w == 0) {
    const size_t cnt = (size_t)(units / w) * unit_elems;
    ncclResult_t r = nccl_lib().all_gather(base + (size_t)c->rank * cnt * elt, base, cnt, t, c->comm, st);
    return r == ncclSuccess ? JULES_OK : nccl_fail(r, "ncclAllGather");
  }
  ncclResult_t r = nccl_lib().group_start();
  for (int q = 0; q < w && r == ncclSuccess; ++q) {
    int64_t b, e;
    jules_dist_shard(units, w, q, &b, &e);
    void* p = base + (size_t)b * unit_elems * elt;
    r = nccl_lib().broadcast(p, p, (size_t)(e - b) * unit_elems, t, q, c->comm, st);
  }
  ncclResult_t r2 = nccl_lib().group_end();
  if (r != ncclSuccess) return nccl_fail(r, "ncclBroadcast");
  return r2 == ncclSuccess ? JULES_OK : nccl_fail(r2, "ncclGroupEnd");
}

}  // namespace
