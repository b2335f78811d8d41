// Shared helpers of libce_b200: status reporting, launch checks and the
// sm_100a PTX wrappers (mbarrier, TMA, tcgen05) used by the tensor-core
// kernels. Every device-side wait here is bounded: it gives up after
// wait_limit_ns() of wall time (read from %globaltimer), records where it
// gave up in a device status word, and returns false so the caller can
// unwind.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <utility>

#include "../../include/ce_b200.h"

namespace ce {

// ---------------------------------------------------------------------------
// Host-side status

// Records msg as the calling thread's last error and returns code.
int set_error(int code, const std::string &msg);
int cuda_error(cudaError_t err, const char *what);
inline int ok() { return CE_OK; }

#define CE_CUDA_TRY(call)                                             \
  do {                                                                \
    cudaError_t ce_err__ = (call);                                    \
    if (ce_err__ != cudaSuccess) return ::ce::cuda_error(ce_err__, #call); \
  } while (0)

#define CE_LAUNCH_CHECK(what) CE_CUDA_TRY(cudaPeekAtLastError())

#define CE_REQUIRE(cond, ...)                                          \
  do {                                                                 \
    if (!(cond)) return ::ce::set_error(CE_ERR_USAGE, ::ce::format(__VA_ARGS__)); \
  } while (0)

std::string format(const char *fmt, ...);

int sm_count();          // SMs of the current device (cached per device)
bool is_sm100();         // compute capability 10.x

// Device status word of the kernels that wait on barriers. Each such .cu
// file owns one as a file-scope __device__ variable; the host reads and
// clears it after synchronizing (ce_device_status in capi.cu).
struct DeviceStatus {
  unsigned int code;    // 0 = fine, else CE_ERR_TIMEOUT
  unsigned int where;   // which wait gave up (site id)
  unsigned int block;   // blockIdx.x of the first failure
  unsigned int pad;
};

// ---------------------------------------------------------------------------
// Device-side helpers

// Wall-time limit of every bounded wait (2 s unless ce_set_wait_limit
// changes it). Each translation unit that includes this header holds its own
// copy on each device; set_wait_limit_here() writes the copy of the unit it
// is compiled into, on the current device.
static __device__ unsigned long long g_wait_limit_ns = 2000000000ull;

__device__ __forceinline__ unsigned long long wait_limit_ns() {
  return *reinterpret_cast<volatile unsigned long long *>(&g_wait_limit_ns);
}

[[maybe_unused]] static int set_wait_limit_here(unsigned long long ns) {
  const cudaError_t e = cudaMemcpyToSymbol(g_wait_limit_ns, &ns, sizeof(ns));
  return e == cudaSuccess ? CE_OK : CE_ERR_CUDA;
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void report_timeout(DeviceStatus *st, unsigned where) {
  if (st != nullptr && atomicCAS(&st->code, 0u, (unsigned)CE_ERR_TIMEOUT) == 0u) {
    st->where = where;
    st->block = blockIdx.x;
  }
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// --- mbarrier --------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}"
               ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}"
               ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Waits until the phase with the given parity has completed. Returns false
// (and records the site) when wait_limit_ns() passes first, or when another
// thread of the grid already reported a failure.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, DeviceStatus *st,
                                          unsigned where) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long start = globaltimer();
  for (uint32_t spin = 1;; ++spin) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((spin & 255u) == 0u) {
      if (globaltimer() - start > wait_limit_ns()) {
        report_timeout(st, where);
        return false;
      }
      if (st != nullptr && *(volatile unsigned *)&st->code != 0u) return false;
    }
  }
}

// Warp-collective bounded wait: every lane polls, the result is the AND over
// the warp, so control flow after it stays warp-uniform (the .aligned
// tcgen05 instructions and barriers that follow need that).
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, DeviceStatus *st,
                                          unsigned where) {
  const bool r = mbar_wait(bar, parity, st, where);
  return __all_sync(0xffffffffu, r) != 0;
}

// --- programmatic dependent launch -------------------------------------------
// A kernel launched with the programmatic-serialization attribute may start
// while its predecessor in the stream still runs. pdl_wait blocks until the
// predecessor has completed and its memory is visible; nothing that reads a
// buffer an earlier kernel writes, or writes a buffer an earlier kernel
// reads, may come before it. pdl_launch_dependents lets the successor start
// its own prologue. Both are no-ops for a kernel launched normally.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// --- peer-memory exchange between ranks (one GPU each) ---------------------
// A producer writes its slice of an exchange into every rank's buffer (its
// own and the peers', mapped by CUDA IPC over NVLink); after its last CTA has
// written, it stores the exchange's epoch into each peer's flag for the
// sending rank. A consumer waits until every peer's flag has reached the
// epoch before it reads. Epoch = generation << 32 | (step * per_step +
// index + 1): the generation advances per run, the step is the device step
// counter, so one captured graph serves every step.
// A GEMM operand in one of the library's stored formats, for
// dequant_operand (quant.cu), which writes it back as fp32 [rows][out_ld].
enum OperandFormat { kOperandF32 = 0, kOperandBF16, kOperandE4M3, kOperandMXFP6, kOperandNVFP4 };
struct DequantOperand {
  int format = kOperandF32;
  const void *data = nullptr;    // elements (fp32 / bf16 / E4M3) or packed bytes
  int ld = 0;                    // row stride: elements, or bytes for MXFP6 / NVFP4
  int rows = 0, cols = 0;
  const float *row_scale = nullptr;     // E4M3: one fp32 per row
  const uint8_t *sf = nullptr;          // block scales: row-major [rows][nsf] or atoms
  bool atoms = false;
  int nsf = 0, katoms = 0, group_rows = 0;
  const float *tensor_decode = nullptr; // NVFP4: the decode tensor scale
  float *out = nullptr;
  int out_ld = 0;
};
int dequant_operand(const DequantOperand &d, cudaStream_t s);

// Extra outputs of the rows launch for the block-scaled GEMMs (rows.cu):
// the MXFP6 packed operand and its scale atoms written from the normalized
// rows, or the max |normalized| for the NVFP4 tensor scale.
struct RowsExtras {
  uint8_t *mx_operand = nullptr;   // [rows][mx_ld bytes]
  int mx_ld = 0;
  uint8_t *mx_atoms = nullptr;     // A-operand UE8M0 scale atoms (128-row groups)
  int katoms = 0;
  unsigned int *amax_bits = nullptr;
  int keep_normalized = 0;         // write the fp32 normalized rows L2-resident
};

struct ExchangeWait {
  const unsigned long long *flags;  // this rank's flags of the exchange kind, one per sending rank; null = no wait
  const unsigned *gen;
  const int *step;
  int world, rank, per_step, index;
};
struct ExchangePut {
  uint8_t *const *blocks;  // every rank's exchange block as mapped here; null = local write only
  size_t flag_off;         // byte offset of flags[kind][this rank] in a block
  int *counter;            // arrival counter of the producer's CTAs (reset by the last)
  const unsigned *gen;
  const int *step;
  int world, rank, per_step, index;
};

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned long long *p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long exchange_epoch(const unsigned *gen, const int *step, int per_step,
                                                             int index) {
  return ((unsigned long long)*gen << 32) | (unsigned)(*step * per_step + index + 1);
}

// Called by one warp: lane q waits (bounded) for peer q's flag. Returns false,
// after recording `where`, if a peer never delivered.
__device__ __forceinline__ bool exchange_wait_warp(const ExchangeWait &w, DeviceStatus *st, unsigned where) {
  const int q = threadIdx.x & 31;
  bool ok = true;
  if (q < w.world && q != w.rank) {
    const unsigned long long epoch = exchange_epoch(w.gen, w.step, w.per_step, w.index);
    unsigned long long start = 0;
    for (uint32_t spin = 1; ld_acquire_sys(w.flags + q) < epoch; ++spin) {
      if ((spin & 1023u) == 0u) {
        const unsigned long long now = globaltimer();
        if (start == 0) {
          start = now;
        } else if (now - start > wait_limit_ns()) {
          report_timeout(st, where);
          ok = false;
          break;
        }
      }
    }
  }
  return __all_sync(0xffffffffu, ok) != 0;
}

// Called by every thread of a producer CTA after its writes: the last CTA of
// the grid to arrive signals the peers. Contains __syncthreads.
__device__ __forceinline__ void exchange_signal(const ExchangePut &p) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(p.counter, 1) == (int)(gridDim.x * gridDim.y * gridDim.z) - 1) {
    *p.counter = 0;
    __threadfence_system();
    const unsigned long long epoch = exchange_epoch(p.gen, p.step, p.per_step, p.index);
    for (int q = 0; q < p.world; ++q)
      if (q != p.rank) st_release_sys(reinterpret_cast<unsigned long long *>(p.blocks[q] + p.flag_off), epoch);
  }
}

// --- row-shard exchange of the op-trio GEMM (rowshard.cu) -------------------
// Rank r of `world` multiplies by its contiguous slice of W's rows; the GEMM's
// epilogue stores each output tile into every rank's [batch][rows] output
// (peer memory mapped by CUDA IPC, plain NVLink stores). Two flags per rank
// pair order the exchange, both in the receiver's block:
//   ready[q]  rank q may be sent exchange e: q's GEMM for e has started, so
//             every consumer of q's exchange e - 1 (earlier on q's stream)
//             is done; a sender waits for it before its first peer store;
//   done[q]   every CTA of q's GEMM for e has stored and fenced; the
//             receiver's rowx_wait_kernel waits for it, then advances its
//             exchange counter (e = counter + 1, in device memory, so a
//             captured graph advances it on every replay).
constexpr int kRowxMaxRanks = 8;
struct RowxSync {
  uint8_t *blocks[kRowxMaxRanks] = {};      // every rank's exchange block as mapped here (own included)
  size_t ready_off = 0, done_off = 0;       // byte offsets of ready[] / done[] (u64 per rank) in a block
  const unsigned long long *epoch = nullptr;  // this rank's count of completed exchanges
  int *counter = nullptr;                   // arrival counter of the GEMM's CTAs (reset by the last)
  int world = 0, rank = 0;                  // world <= 1: no fan-out
};

__device__ __forceinline__ unsigned long long rowx_exchange(const RowxSync &rx) {
  return *reinterpret_cast<const volatile unsigned long long *>(rx.epoch) + 1ull;
}

// One thread per CTA of the sending GEMM, after its launch wait: tells every
// peer that this rank accepts exchange e (idempotent; every CTA sends it, so
// no CTA's progress depends on another being resident).
__device__ __forceinline__ void rowx_signal_ready(const RowxSync &rx) {
  const unsigned long long e = rowx_exchange(rx);
  for (int q = 0; q < rx.world; ++q)
    if (q != rx.rank)
      st_release_sys(reinterpret_cast<unsigned long long *>(rx.blocks[q] + rx.ready_off) + rx.rank, e);
}

// One warp: lane q waits (bounded) until peer q accepts exchange e.
__device__ __forceinline__ bool rowx_wait_ready_warp(const RowxSync &rx, DeviceStatus *st, unsigned where) {
  const int q = threadIdx.x & 31;
  bool ok = true;
  if (q < rx.world && q != rx.rank) {
    const unsigned long long e = rowx_exchange(rx);
    const unsigned long long *flag =
        reinterpret_cast<const unsigned long long *>(rx.blocks[rx.rank] + rx.ready_off) + q;
    unsigned long long start = 0;
    for (uint32_t spin = 1; ld_acquire_sys(flag) < e; ++spin) {
      if ((spin & 1023u) == 0u) {
        const unsigned long long now = globaltimer();
        if (start == 0) {
          start = now;
        } else if (now - start > wait_limit_ns()) {
          report_timeout(st, where);
          ok = false;
          break;
        }
      }
    }
  }
  return __all_sync(0xffffffffu, ok) != 0;
}

// Every thread of every CTA of the sending GEMM, after its last store: the
// last CTA to arrive tells every peer that exchange e has landed. Contains
// __syncthreads.
__device__ __forceinline__ void rowx_signal_done(const RowxSync &rx) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned long long e = rowx_exchange(rx);
    if (atomicAdd(rx.counter, 1) == (int)(gridDim.x * gridDim.y * gridDim.z) - 1) {
      *rx.counter = 0;
      __threadfence_system();
      for (int q = 0; q < rx.world; ++q)
        if (q != rx.rank)
          st_release_sys(reinterpret_cast<unsigned long long *>(rx.blocks[q] + rx.done_off) + rx.rank, e);
    }
  }
}

// --- clusters (CTA pairs of the 2-SM tensor-core path) ---------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same shared-memory offset in CTA `rank`.
__device__ __forceinline__ uint32_t cluster_map(uint32_t local_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}
// Arrive on an mbarrier of any CTA of the cluster (shared::cluster address).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];"
               ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx_cluster(uint32_t cluster_addr, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cluster.shared::cluster.b64 _, [%0], %1;"
               ::"r"(cluster_addr), "r"(bytes) : "memory");
}
// try_wait with cluster-scope acquire, for barriers that other CTAs of the
// cluster arrive on.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t *bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t *bar, uint32_t parity, DeviceStatus *st,
                                                  unsigned where) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const unsigned long long start = globaltimer();
  for (uint32_t spin = 1;; ++spin) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((spin & 255u) == 0u) {
      if (globaltimer() - start > wait_limit_ns()) {
        report_timeout(st, where);
        return false;
      }
      if (st != nullptr && *(volatile unsigned *)&st->code != 0u) return false;
    }
  }
}
__device__ __forceinline__ bool warp_wait_cluster(uint64_t *bar, uint32_t parity, DeviceStatus *st,
                                                  unsigned where) {
  const bool r = mbar_wait_cluster(bar, parity, st, where);
  return __all_sync(0xffffffffu, r) != 0;
}

// --- TMA -------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const void *desc) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(desc) : "memory");
}

// 2-D tiled bulk tensor load into this CTA's shared memory, completion
// signalled on bar (no multicast).
__device__ __forceinline__ void tma_load_2d(void *smem_dst, const void *desc, uint64_t *bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(smem_dst)), "l"(desc), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// Prefetch of a 2-D tile into L2 (no shared memory written, no barrier).
__device__ __forceinline__ void tma_prefetch_2d(const void *desc, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];"
               ::"l"(desc), "r"(x), "r"(y) : "memory");
}

// 2-D tiled load of the CTA-pair form: data lands in this CTA's shared
// memory, completion is signalled on an mbarrier that may belong to the peer
// CTA of the pair (shared::cluster address). No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void *smem_dst, const void *desc,
                                                 uint32_t bar_cluster_addr, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(smem_dst)), "l"(desc), "r"(bar_cluster_addr), "r"(x), "r"(y)
      : "memory");
}

// --- tcgen05 ---------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
               ::"r"(smem_u32(dst_smem)), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
               ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Arrives on bar once every tcgen05.mma issued so far by this thread has
// completed (their shared-memory reads included).
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               ::"r"(smem_u32(bar)) : "memory");
}

// CTA-pair (cta_group::2) forms: allocation and release are issued by the
// same warp in both CTAs of the pair; the MMA and its commits by one thread
// of the even CTA.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
               ::"r"(smem_u32(dst_smem)), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;"
               ::"r"(taddr), "r"(ncols) : "memory");
}
// Arrives on the mbarrier at a shared::cluster address (either CTA of the
// pair) when all prior tcgen05 operations of this thread have completed.
__device__ __forceinline__ void tc_commit_pair(uint32_t bar_cluster_addr) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               ::"r"(bar_cluster_addr) : "memory");
}
template <int kKind>  // 0, 3: kind::f16 (bf16 / fp16 operands), 1: kind::tf32, 2: kind::f8f6f4
__device__ __forceinline__ void tc_mma_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  if constexpr (kKind == 0 || kKind == 3) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
  } else if constexpr (kKind == 1) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
  } else {
    static_assert(kKind == 2, "unknown MMA kind");
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
  }
}

// D(tmem) (+)= A(smem desc) x B(smem desc)^T, one instruction.
template <int kKind>  // 0, 3: kind::f16 (bf16 / fp16 operands), 1: kind::tf32, 2: kind::f8f6f4
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  if constexpr (kKind == 0 || kKind == 3) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
  } else if constexpr (kKind == 1) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
  } else {
    static_assert(kKind == 2, "unknown MMA kind");
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
  }
}

// 32 lanes x 32 consecutive fp32 columns per warp: thread t of the warp gets
// lane (base lane + t), columns [col, col + 32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}
// 32 lanes x 16 consecutive fp32 columns per warp (as the x32 form).
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// 32 lanes x 32 consecutive 32-bit columns per warp, from registers.
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]),
        "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
        "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
        "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
        "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// D(tmem) (+)= A(tmem) x B(smem desc)^T, kind::f16, one instruction. A in
// tensor memory: lane = row, column = k / 2 (two 16-bit values per column,
// the even k in the low half).
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// Makes this thread's generic-proxy shared-memory writes visible to the
// async proxy (the tensor cores and bulk copies read through it).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Shared-memory matrix descriptor of a K-major operand tile stored with the
// 128-byte swizzle (rows of 128 bytes, 8-row / 1024-byte swizzle atoms):
// start address >> 4 in bits 0-13, leading byte offset (unused by swizzled
// K-major layouts, encoded as 1) in bits 16-29, stride byte offset (1024 B
// between 8-row groups) >> 4 in bits 32-45, descriptor version 1 in bits
// 46-47, base offset 0 (atoms are 1024-byte aligned), layout type 2
// (SWIZZLE_128B) in bits 61-63.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

// Descriptor of an MN-major operand tile with the 128-byte swizzle: 64
// consecutive MN elements (128 bytes) per K row, 8 K rows per 1024-byte
// atom; lbo = bytes between successive 64-element MN chunks, 1024 bytes
// between successive 8-row K groups (the canonical MN-major SW128 layout,
// which a TMA load of a [K rows][64 elements] box with SWIZZLE_128B writes).
__device__ __forceinline__ uint64_t smem_desc_sw128_mn(uint32_t smem_addr, uint32_t lbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

// Launches kernel<<<grid, block, smem, s>>>(args...), with programmatic
// stream serialization when pdl is set (the kernel must call pdl_wait before
// touching memory that earlier kernels use).
template <typename... KArgs, typename... Args>
int launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                  bool pdl, const char *what, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = pdl ? attr : nullptr;
  cfg.numAttrs = pdl ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  return e == cudaSuccess ? CE_OK : cuda_error(e, what);
}

}  // namespace ce

