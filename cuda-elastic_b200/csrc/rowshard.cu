// Row-shard (tensor-parallel) layer of the op-trio GEMM across the GPUs of
// one node. The reference runs the classifier GEMM on one GPU
// (applications/loom_private/decoder/decoder.cu:83-125,
// experiments/blackwell/lowprec/decoder_lowprec.cu:85-127); here W's rows
// are split into contiguous slices, rank r of n multiplies the full
// normalized batch by rows [lo_r, hi_r), and the slices are joined into
// every rank's out[batch][rows] in one of two ways:
//   * NCCL (ce_allgather_rows): each rank's GEMM writes its slice into its
//     slot of a [world][batch][width] staging buffer, ncclAllGather (in
//     place) gives every rank all slots, and join_rows_kernel scatters the
//     slots into the row-major output. NCCL is resolved at run time from the
//     libnccl.so.2 the process has already loaded (PyTorch's, or the one a
//     C++ host links), so the caller's communicator and this library use the
//     same NCCL.
//   * peer memory (ce_rowx_*, ce_plan_gemm_rowx): every rank's output lives
//     in an exchange block shared by CUDA IPC; the GEMM's epilogue stores
//     each tile into all ranks' blocks over NVLink as it leaves tensor
//     memory, so the exchange overlaps the multiply tile by tile and needs
//     no join kernel. Flags order it (RowxSync, common.cuh); every wait is
//     bounded and reported through ce_device_status.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace ce {

static __device__ DeviceStatus g_rowx_status;

int rowx_set_wait_limit(unsigned long long ns) { return set_wait_limit_here(ns); }

int rowx_status() {
  CE_CUDA_TRY(cudaDeviceSynchronize());
  DeviceStatus h{};
  CE_CUDA_TRY(cudaMemcpyFromSymbol(&h, g_rowx_status, sizeof(h)));
  if (h.code == 0) return CE_OK;
  const DeviceStatus zero{};
  CE_CUDA_TRY(cudaMemcpyToSymbol(g_rowx_status, &zero, sizeof(zero)));
  return set_error(CE_ERR_TIMEOUT, format("row-shard exchange wait gave up (site %u): a peer never delivered", h.where));
}

namespace {

// One warp: lane q waits (bounded) until peer q's GEMM for the next exchange
// has stored its slice here; then the exchange counter advances.
__global__ void rowx_wait_kernel(const unsigned long long *done, unsigned long long *epoch, int world, int rank) {
  const int q = threadIdx.x;
  const unsigned long long e = *reinterpret_cast<volatile unsigned long long *>(epoch) + 1ull;
  if (q < world && q != rank) {
    const unsigned long long start = globaltimer();
    for (uint32_t spin = 1; ld_acquire_sys(done + q) < e; ++spin) {
      if ((spin & 255u) == 0u && globaltimer() - start > wait_limit_ns()) {
        report_timeout(&g_rowx_status, 80u);
        break;
      }
    }
  }
  // advanced even after a timeout (reported above), so the ranks' counters
  // stay in step with the flags the peers go on sending
  __syncwarp();
  if (q == 0) *epoch = e;
}

// First step of ce_rowx_put, one warp: tells every peer that this rank
// accepts the next exchange (its consumers of the previous one ran earlier
// in the stream), then lane q waits (bounded) until peer q accepts it too.
__global__ void rowx_ready_kernel(RowxSync rx) {
  if (threadIdx.x == 0) rowx_signal_ready(rx);
  rowx_wait_ready_warp(rx, &g_rowx_status, 81u);
}

// Last step of ce_rowx_put: the copies before it in the stream have landed
// in the peers' blocks; tell every peer.
__global__ void rowx_done_kernel(RowxSync rx) {
  __threadfence_system();
  const unsigned long long e = rowx_exchange(rx);
  for (int q = 0; q < rx.world; ++q)
    if (q != rx.rank)
      st_release_sys(reinterpret_cast<unsigned long long *>(rx.blocks[q] + rx.done_off) + rx.rank, e);
}

// out[b][c] = staging[q][b][c - lo_q] for the rank q whose slice holds
// column c (bounds of shard_bounds); one thread per 4 outputs when the
// slices are 4-aligned, else per output.
__global__ void join_rows_kernel(float *out, const float *staging, int batch, int rows, int world, int width) {
  const int base = rows / world, extra = rows % world;
  const long long total = (long long)batch * rows;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int b = (int)(i / rows), c = (int)(i - (long long)b * rows);
    // rank of column c: the first `extra` ranks hold base + 1 columns
    const int big = extra * (base + 1);
    const int q = c < big ? c / (base + 1) : extra + (c - big) / base;
    const int lo = q * base + (q < extra ? q : extra);
    out[i] = staging[((size_t)q * batch + b) * width + (c - lo)];
  }
}

__global__ void join_rows_vec_kernel(float4 *out, const float4 *staging, int batch, int rows4, int width4) {
  // every slice is width4 float4 columns wide (rows % (4 * world) == 0)
  const long long total = (long long)batch * rows4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int b = (int)(i / rows4), c = (int)(i - (long long)b * rows4);
    const int q = c / width4;
    out[i] = staging[((size_t)q * batch + b) * width4 + (c - q * width4)];
  }
}

// --- NCCL, resolved at run time ---------------------------------------------
struct NcclApi {
  ncclResult_t (*get_version)(int *);
  ncclResult_t (*get_unique_id)(ncclUniqueId *);
  ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int);
  ncclResult_t (*comm_destroy)(ncclComm_t);
  ncclResult_t (*comm_count)(const ncclComm_t, int *);
  ncclResult_t (*comm_user_rank)(const ncclComm_t, int *);
  ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
  const char *(*error_string)(ncclResult_t);
  bool ok = false;
};

// Binds to the libnccl.so.2 the process has already loaded (the caller's
// NCCL: PyTorch's, or the one a C++ host links), never to another copy: two
// NCCLs of the same soname in one process would shadow each other's symbols.
// Until the caller has loaded one, every call fails and the next one retries.
const NcclApi &nccl() {
  static NcclApi api;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  if (!api.ok) {
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (h == nullptr) return api;
    api.get_version = reinterpret_cast<decltype(api.get_version)>(dlsym(h, "ncclGetVersion"));
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    api.comm_count = reinterpret_cast<decltype(api.comm_count)>(dlsym(h, "ncclCommCount"));
    api.comm_user_rank = reinterpret_cast<decltype(api.comm_user_rank)>(dlsym(h, "ncclCommUserRank"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
    api.ok = api.get_version && api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.comm_count &&
             api.comm_user_rank && api.all_gather && api.error_string;
  }
  return api;
}

int nccl_error(ncclResult_t r, const char *what) {
  return set_error(CE_ERR_CUDA, format("%s failed: %s", what, nccl().error_string ? nccl().error_string(r) : "?"));
}

#define CE_NCCL_REQUIRE()                                                                          \
  do {                                                                                             \
    if (!nccl().ok) return set_error(CE_ERR_USAGE, "no libnccl.so.2 is loaded in this process");   \
  } while (0)

void shard_range(int rows, int world, int rank, int *lo, int *hi) {
  const int base = rows / world, extra = rows % world;
  *lo = rank * base + (rank < extra ? rank : extra);
  *hi = *lo + base + (rank < extra ? 1 : 0);
}

}  // namespace
}  // namespace ce

using namespace ce;

// Exchange block of one rank: out [batch][rows] fp32, then ready[8] and
// done[8] (u64, written by the peers). The exchange counter and the GEMM's
// CTA arrival counter live apart in memory no peer maps.
struct ce_rowx {
  int batch = 0, rows = 0, world = 0, rank = 0, device = 0;
  int lo = 0, hi = 0;
  uint8_t *block = nullptr;
  size_t out_bytes = 0, ready_off = 0, done_off = 0, block_bytes = 0;
  unsigned long long *local = nullptr;  // [0] exchange counter, [1] arrival counter (int)
  uint8_t *peer[kRowxMaxRanks] = {};
  bool connected = false;
  // ce_rowx_put: one stream per peer so the copies run on several copy
  // engines at once, forked from and joined back to the caller's stream
  cudaStream_t cs[kRowxMaxRanks] = {};
  cudaEvent_t fork = nullptr, join[kRowxMaxRanks] = {};
};

namespace ce {
int x_device_of(const ce_rowx *x) { return x->device; }

// Fills the GEMM's view of an exchange (used by ce_plan_gemm_rowx).
int rowx_sync(const ce_rowx *x, RowxSync *rx, float **out, int *lo, int *hi, int *batch, int *rows) {
  CE_REQUIRE(x != nullptr, "null row-shard exchange");
  CE_REQUIRE(x->connected, "the row-shard exchange is not connected (ce_rowx_connect)");
  int dev = 0;
  CE_CUDA_TRY(cudaGetDevice(&dev));
  CE_REQUIRE(dev == x->device, "the row-shard exchange belongs to device %d, current device is %d", x->device, dev);
  for (int q = 0; q < kRowxMaxRanks; ++q) rx->blocks[q] = q < x->world ? x->peer[q] : nullptr;
  rx->ready_off = x->ready_off;
  rx->done_off = x->done_off;
  rx->epoch = x->local;
  rx->counter = reinterpret_cast<int *>(x->local + 1);
  rx->world = x->world;
  rx->rank = x->rank;
  *out = reinterpret_cast<float *>(x->block);
  *lo = x->lo;
  *hi = x->hi;
  *batch = x->batch;
  *rows = x->rows;
  return CE_OK;
}
}  // namespace ce

extern "C" {

int ce_shard_bounds(int rows, int world, int rank, int *lo, int *hi) {
  CE_REQUIRE(lo != nullptr && hi != nullptr, "null output");
  CE_REQUIRE(rows >= 1 && world >= 1 && rank >= 0 && rank < world, "bad shard (rows %d, world %d, rank %d)",
             rows, world, rank);
  shard_range(rows, world, rank, lo, hi);
  return CE_OK;
}

int ce_rowx_open(ce_rowx **out, int batch, int rows, int world, int rank, void *handle_out) {
  CE_REQUIRE(out != nullptr && handle_out != nullptr, "null argument");
  *out = nullptr;
  CE_REQUIRE(batch >= 1 && rows >= 1, "batch and rows must be >= 1");
  CE_REQUIRE(world >= 2 && world <= kRowxMaxRanks, "the row-shard exchange needs 2..%d ranks (got %d)",
             kRowxMaxRanks, world);
  CE_REQUIRE(rank >= 0 && rank < world, "rank %d is outside world %d", rank, world);
  CE_REQUIRE(rows >= world, "fewer rows (%d) than ranks (%d)", rows, world);
  ce_rowx *x = new ce_rowx();
  x->batch = batch;
  x->rows = rows;
  x->world = world;
  x->rank = rank;
  shard_range(rows, world, rank, &x->lo, &x->hi);
  x->out_bytes = (((size_t)batch * rows * 4) + 255) / 256 * 256;
  x->ready_off = x->out_bytes;
  x->done_off = x->ready_off + 8 * kRowxMaxRanks;
  x->block_bytes = x->done_off + 8 * kRowxMaxRanks;
  cudaError_t e = cudaGetDevice(&x->device);
  if (e == cudaSuccess) e = cudaMalloc(&x->block, x->block_bytes);
  if (e == cudaSuccess) e = cudaMalloc(&x->local, 2 * sizeof(unsigned long long));
  if (e == cudaSuccess) e = cudaMemset(x->block, 0, x->block_bytes);
  if (e == cudaSuccess) e = cudaMemset(x->local, 0, 2 * sizeof(unsigned long long));
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&x->fork, cudaEventDisableTiming);
  for (int q = 0; q < world && e == cudaSuccess; ++q) {
    if (q == rank) continue;
    e = cudaStreamCreateWithFlags(&x->cs[q], cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&x->join[q], cudaEventDisableTiming);
  }
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, x->block);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    ce_rowx_close(x);
    return cuda_error(e, "ce_rowx_open");
  }
  static_assert(sizeof(cudaIpcMemHandle_t) <= CE_IPC_HANDLE_BYTES, "IPC handle size");
  memset(handle_out, 0, CE_IPC_HANDLE_BYTES);
  memcpy(handle_out, &h, sizeof(h));
  x->peer[rank] = x->block;
  *out = x;
  return CE_OK;
}

int ce_rowx_connect(ce_rowx *x, const void *handles) {
  CE_REQUIRE(x != nullptr && handles != nullptr, "null argument");
  CE_REQUIRE(!x->connected, "the row-shard exchange is already connected");
  for (int q = 0; q < x->world; ++q) {
    if (q == x->rank) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, static_cast<const uint8_t *>(handles) + (size_t)q * CE_IPC_HANDLE_BYTES, sizeof(h));
    void *p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_error(e, format("cudaIpcOpenMemHandle(rank %d)", q).c_str());
    x->peer[q] = static_cast<uint8_t *>(p);
  }
  x->connected = true;
  return CE_OK;
}

int ce_rowx_output(ce_rowx *x, float **out_dev, int *lo, int *hi) {
  CE_REQUIRE(x != nullptr && out_dev != nullptr, "null argument");
  *out_dev = reinterpret_cast<float *>(x->block);
  if (lo) *lo = x->lo;
  if (hi) *hi = x->hi;
  return CE_OK;
}

int ce_rowx_wait(ce_rowx *x, ce_stream_t stream) {
  CE_REQUIRE(x != nullptr, "null row-shard exchange");
  // needs only this rank's own block: the peers' done flags land in it
  const unsigned long long *done = reinterpret_cast<const unsigned long long *>(x->block + x->done_off);
  return launch_kernel(rowx_wait_kernel, dim3(1), dim3(32), 0, (cudaStream_t)stream, false, "rowx_wait_kernel",
                       done, x->local, x->world, x->rank);
}

int ce_rowx_put(ce_rowx *x, ce_stream_t stream) {
  RowxSync rx;
  float *out = nullptr;
  int lo = 0, hi = 0, batch = 0, rows = 0;
  int rc = rowx_sync(x, &rx, &out, &lo, &hi, &batch, &rows);
  if (rc) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  rc = launch_kernel(rowx_ready_kernel, dim3(1), dim3(32), 0, s, false, "rowx_ready_kernel", rx);
  if (rc) return rc;
  // this rank's columns [lo, hi) of every row, to the same place in each
  // peer's block: strided copies over NVLink, one per peer on its own
  // stream so several copy engines work at once
  const size_t pitch = (size_t)rows * 4, off = (size_t)lo * 4;
  CE_CUDA_TRY(cudaEventRecord(x->fork, s));
  for (int q = 0; q < x->world; ++q) {
    if (q == x->rank) continue;
    CE_CUDA_TRY(cudaStreamWaitEvent(x->cs[q], x->fork, 0));
    CE_CUDA_TRY(cudaMemcpy2DAsync(x->peer[q] + off, pitch, x->block + off, pitch, (size_t)(hi - lo) * 4, batch,
                                  cudaMemcpyDeviceToDevice, x->cs[q]));
    CE_CUDA_TRY(cudaEventRecord(x->join[q], x->cs[q]));
    CE_CUDA_TRY(cudaStreamWaitEvent(s, x->join[q], 0));
  }
  return launch_kernel(rowx_done_kernel, dim3(1), dim3(1), 0, s, false, "rowx_done_kernel", rx);
}

int ce_rowx_close(ce_rowx *x) {
  if (x == nullptr) return CE_OK;
  for (int q = 0; q < x->world; ++q) {
    if (x->cs[q] != nullptr) cudaStreamSynchronize(x->cs[q]);
    if (q != x->rank && x->peer[q] != nullptr) cudaIpcCloseMemHandle(x->peer[q]);
    if (x->cs[q] != nullptr) cudaStreamDestroy(x->cs[q]);
    if (x->join[q] != nullptr) cudaEventDestroy(x->join[q]);
  }
  if (x->fork) cudaEventDestroy(x->fork);
  if (x->block) cudaFree(x->block);
  if (x->local) cudaFree(x->local);
  delete x;
  return CE_OK;
}

int ce_nccl_version(int *version) {
  CE_REQUIRE(version != nullptr, "null argument");
  *version = 0;
  CE_NCCL_REQUIRE();
  const ncclResult_t r = nccl().get_version(version);
  return r == ncclSuccess ? CE_OK : nccl_error(r, "ncclGetVersion");
}

int ce_nccl_unique_id(void *id_out) {
  CE_REQUIRE(id_out != nullptr, "null argument");
  CE_NCCL_REQUIRE();
  static_assert(sizeof(ncclUniqueId) == CE_NCCL_ID_BYTES, "NCCL unique id size");
  ncclUniqueId id;
  const ncclResult_t r = nccl().get_unique_id(&id);
  if (r != ncclSuccess) return nccl_error(r, "ncclGetUniqueId");
  memcpy(id_out, &id, sizeof(id));
  return CE_OK;
}

int ce_nccl_comm_init(void **comm_out, int world, int rank, const void *id) {
  CE_REQUIRE(comm_out != nullptr && id != nullptr, "null argument");
  *comm_out = nullptr;
  CE_REQUIRE(world >= 1 && rank >= 0 && rank < world, "rank %d is outside world %d", rank, world);
  CE_NCCL_REQUIRE();
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  ncclComm_t c = nullptr;
  const ncclResult_t r = nccl().comm_init_rank(&c, world, uid, rank);
  if (r != ncclSuccess) return nccl_error(r, "ncclCommInitRank");
  *comm_out = c;
  return CE_OK;
}

int ce_nccl_comm_destroy(void *comm) {
  if (comm == nullptr) return CE_OK;
  CE_NCCL_REQUIRE();
  const ncclResult_t r = nccl().comm_destroy(static_cast<ncclComm_t>(comm));
  return r == ncclSuccess ? CE_OK : nccl_error(r, "ncclCommDestroy");
}

int ce_allgather_staging_floats(int batch, int rows, int world, size_t *floats) {
  CE_REQUIRE(floats != nullptr, "null argument");
  CE_REQUIRE(batch >= 1 && rows >= 1 && world >= 1 && rows >= world, "bad shape (batch %d, rows %d, world %d)",
             batch, rows, world);
  *floats = (size_t)world * batch * ((rows + world - 1) / world);
  return CE_OK;
}

int ce_allgather_rows(void *comm, float *out, float *staging, int batch, int rows, int world, int rank,
                      ce_stream_t stream) {
  CE_REQUIRE(comm != nullptr && out != nullptr && staging != nullptr, "null argument");
  CE_REQUIRE(batch >= 1 && rows >= world && world >= 1 && rank >= 0 && rank < world,
             "bad shape (batch %d, rows %d, world %d, rank %d)", batch, rows, world, rank);
  CE_NCCL_REQUIRE();
  int n = 0, r = 0;
  ncclResult_t nr = nccl().comm_count(static_cast<ncclComm_t>(comm), &n);
  if (nr == ncclSuccess) nr = nccl().comm_user_rank(static_cast<ncclComm_t>(comm), &r);
  if (nr != ncclSuccess) return nccl_error(nr, "ncclCommCount / ncclCommUserRank");
  CE_REQUIRE(n == world && r == rank, "communicator is rank %d of %d, the call says rank %d of %d", r, n, rank, world);
  cudaStream_t s = (cudaStream_t)stream;
  const int width = (rows + world - 1) / world;
  const size_t slot = (size_t)batch * width;
  if (world > 1) {
    nr = nccl().all_gather(staging + (size_t)rank * slot, staging, slot, ncclFloat32, static_cast<ncclComm_t>(comm), s);
    if (nr != ncclSuccess) return nccl_error(nr, "ncclAllGather");
  }
  const long long total = (long long)batch * rows;
  const bool vec = rows % (4 * world) == 0 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0 &&
                   (reinterpret_cast<uintptr_t>(staging) & 15u) == 0;
  const int threads = 256;
  const long long work = vec ? total / 4 : total;
  const int grid = (int)std::min<long long>((work + threads - 1) / threads, (long long)sm_count() * 8);
  if (vec)
    return launch_kernel(join_rows_vec_kernel, dim3(grid), dim3(threads), 0, s, false, "join_rows_vec_kernel",
                         reinterpret_cast<float4 *>(out), reinterpret_cast<const float4 *>(staging), batch,
                         rows / 4, width / 4);
  return launch_kernel(join_rows_kernel, dim3(grid), dim3(threads), 0, s, false, "join_rows_kernel", out,
                       (const float *)staging, batch, rows, world, width);
}

}  // extern "C"
