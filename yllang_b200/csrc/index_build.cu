// Batch index build for sm_100a: from per-sequence lengths and page-table rows
// produce kv_indptr / kv_indices / kv_last_page_len / qo_indptr / slot_mapping.
//
// The reference builds its per-step indices on the host, one libtorch scalar
// op per element (Make2DIndices, src/include/batch/batch_manager.h:30-51,
// called from NextBatch, batch_manager.h:97-112), for page size 1.  Here the
// whole batch is one launch:
//
//   phase A  every block redundantly computes each sequence's page count and
//            new-token count and exclusive-scans both into shared memory
//            (B <= kSmemBatchLimit; the batch is a few KB, an L2 hit for every
//            block after the first, so this avoids any inter-block handshake);
//   phase B  the blocks write kv_indptr, qo_indptr and kv_last_page_len;
//   phase C  the concatenated element space [kv_indices | slot_mapping] is cut
//            into equal contiguous chunks, one per block; each thread finds its
//            element's sequence by binary search over the scanned offsets and
//            gathers from that sequence's page-table row, so reads of a row and
//            writes of kv_indices are both coalesced.
//
// Batches above kSmemBatchLimit take a two-launch form: one block scans into
// the kv_indptr / qo_indptr outputs, then the fill reads them from global
// memory.  Neither form needs memory beyond the caller's outputs.
#include <cuda_runtime.h>

#include <climits>
#include <cstdint>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "index_device.cuh"

namespace ylk {

constexpr int kIndexThreads = 256;     // small batches: many blocks, cheap redundant scans
constexpr int kIndexThreadsBig = 1024; // batches above kBigBatch: 4x fewer blocks repeat the scan, loads batched
constexpr int kBigBatch = 512;
constexpr int kScanThreads = 1024;     // one-block scan of the two-launch form
constexpr int kSmemBatchLimit = 16384;
constexpr int kFillUnroll = 4;          // fill elements in flight per thread in the big-batch kernels

// Single-launch form (B <= kSmemBatchLimit).
// kBig: batched staging and the choice of the warp-per-sequence fill (the
// 1024-thread kernel; the 256-thread one too when it runs beside the store).
template <int THREADS, bool kBig = (THREADS == 1024)>
__global__ void __launch_bounds__(THREADS) build_index_kernel(const __grid_constant__ IndexParams p) {
  extern __shared__ int64_t smem[];
  int64_t *scratch = smem;                                   // kScanScratch x int64
  int32_t *kvp = reinterpret_cast<int32_t *>(smem + kScanScratch);  // [B+1]
  int32_t *qop = kvp + (p.batch + 1);                        // [B+1]
  const bool report = blockIdx.x == 0;
  // Launched as a programmatic dependent, wait for the kernel before this one
  // (it may have written the lengths or the page table) before reading
  // anything; then a store launched as our dependent may start loading its
  // K/V rows.  For a normal launch the wait returns at once.
  pdl_wait();
  pdl_trigger();
  if (!scan_batch<kBig>(p, kvp, qop, scratch, report)) return;
  write_seq_outputs(p, kvp, qop, static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x,
                    static_cast<int64_t>(gridDim.x) * blockDim.x, true);
  if constexpr (kBig)
    fill_block_share<kFillUnroll>(p, kvp, qop, report, fill_by_sequence_suits(p, kvp, scanned_max_pages(scratch)));
  else
    fill_block_share<1>(p, kvp, qop, report);
}

// Two-launch form, launch 1 (one block): scan straight into the outputs.  On
// overflow kv_indptr[B] is set to -1 so that launch 2 skips the fill.
__global__ void __launch_bounds__(kScanThreads) scan_index_kernel(const __grid_constant__ IndexParams p) {
  __shared__ int64_t scratch[kScanScratch];
  if (!scan_batch<true>(p, p.kv_indptr, p.qo_indptr, scratch, true)) {
    if (threadIdx.x == 0) p.kv_indptr[p.batch] = -1;
    return;
  }
  write_seq_outputs(p, p.kv_indptr, p.qo_indptr, threadIdx.x, blockDim.x, false);
}

// Two-launch form, launch 2: fill from the scanned outputs.
__global__ void __launch_bounds__(kIndexThreadsBig) fill_index_kernel(const __grid_constant__ IndexParams p) {
  pdl_trigger();
  if (p.kv_indptr[p.batch] < 0) return;
  // the batch's largest page count, from the scanned offsets (each block
  // reads them once, kStageUnroll per thread in flight)
  __shared__ int32_t s_max;
  if (threadIdx.x == 0) s_max = 0;
  __syncthreads();
  int32_t mx = 0;
  for (int base = threadIdx.x; base < p.batch; base += kStageUnroll * blockDim.x) {
    int32_t d[kStageUnroll];
#pragma unroll
    for (int u = 0; u < kStageUnroll; ++u) {
      const int i = base + u * static_cast<int>(blockDim.x);
      d[u] = i < p.batch ? __ldg(p.kv_indptr + i + 1) - __ldg(p.kv_indptr + i) : 0;
    }
#pragma unroll
    for (int u = 0; u < kStageUnroll; ++u) mx = max(mx, d[u]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) atomicMax(&s_max, mx);
  __syncthreads();
  fill_block_share<kFillUnroll>(p, p.kv_indptr, p.qo_indptr, blockIdx.x == 0,
                                fill_by_sequence_suits(p, p.kv_indptr, s_max));
}

static size_t single_launch_smem(int batch) { return kScanScratch * sizeof(int64_t) + 2 * (batch + 1) * sizeof(int32_t); }

// Opt the single-launch kernel into > 48 KB dynamic shared memory once per device.
static int ensure_smem_attr() {
  static std::mutex mu;
  static std::vector<char> done;
  const int dev = current_device();
  std::lock_guard<std::mutex> lock(mu);
  if (static_cast<int>(done.size()) <= dev) done.resize(dev + 1, 0);
  if (!done[dev]) {
    // No carveout preference: the store kernel that runs as this kernel's PDL
    // dependent takes the default split too, so both fit on one SM at once (a
    // differing preference keeps the store's blocks off an SM until it drains).
    cudaError_t e = cudaFuncSetAttribute(build_index_kernel<kIndexThreads>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(single_launch_smem(kSmemBatchLimit)));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(build_index_kernel<kIndexThreadsBig>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(single_launch_smem(kSmemBatchLimit)));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(build_index_kernel<kIndexThreads, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(single_launch_smem(kSmemBatchLimit)));
    if (e != cudaSuccess) {
      set_last_error(std::string("yl_build_index: cudaFuncSetAttribute: ") + cudaGetErrorString(e));
      return YL_ERR_CUDA;
    }
    done[dev] = 1;
  }
  return YL_OK;
}

int prepare_index(const yl_index_args *a, IndexParams &p) {
  if (a == nullptr) return fail(YL_ERR_NULL_ARG, "yl_build_index: args is NULL");
  if (a->batch_size < 0) return fail(YL_ERR_BAD_SIZE, "yl_build_index: batch_size=%lld < 0", a->batch_size);
  if (a->page_size < 1) return fail(YL_ERR_BAD_SIZE, "yl_build_index: page_size=%lld < 1", a->page_size);
  if (a->max_pages_per_row < 0)
    return fail(YL_ERR_BAD_SIZE, "yl_build_index: max_pages_per_row=%lld < 0", a->max_pages_per_row);
  if (a->kv_indices_capacity < 0 || a->slot_capacity < 0)
    return fail(YL_ERR_BAD_SIZE, "yl_build_index: negative capacity (%lld, %lld)", a->kv_indices_capacity,
                a->slot_capacity);
  if (a->slot_is_int64 != 0 && a->slot_is_int64 != 1)
    return fail(YL_ERR_BAD_SIZE, "yl_build_index: slot_is_int64=%lld must be 0 or 1", a->slot_is_int64);
  if (!a->kv_indptr || !a->qo_indptr)
    return fail(YL_ERR_NULL_ARG, "yl_build_index: kv_indptr and qo_indptr are required");
  if (a->batch_size > 0 && (!a->prior_len || !a->new_len))
    return fail(YL_ERR_NULL_ARG, "yl_build_index: prior_len and new_len are required");
  const bool wants_gather = (a->kv_indices && a->kv_indices_capacity > 0) || (a->slot_mapping && a->slot_capacity > 0);
  if (a->batch_size > 0 && wants_gather && !a->page_table)
    return fail(YL_ERR_NULL_ARG, "yl_build_index: page_table is required for kv_indices / slot_mapping");
  if (a->table_index && a->num_table_rows <= 0)
    return fail(YL_ERR_BAD_SIZE, "yl_build_index: num_table_rows=%lld must be > 0 with table_index",
                a->num_table_rows);
  if (!a->table_index && a->num_table_rows > 0 && a->num_table_rows < a->batch_size)
    return fail(YL_ERR_BAD_SIZE, "yl_build_index: %lld page-table rows for a batch of %lld", a->num_table_rows,
                a->batch_size);
  if (a->page_table_stride < 0)
    return fail(YL_ERR_BAD_SIZE, "yl_build_index: page_table_stride=%lld < 0", a->page_table_stride);
  if ((a->kv_indices ? a->kv_indices_capacity : 0) + (a->slot_mapping ? a->slot_capacity : 0) >= (1ll << 31))
    return fail(YL_ERR_UNSUPPORTED, "yl_build_index: kv_indices + slot capacity of %lld elements reaches 2^31",
                (a->kv_indices ? a->kv_indices_capacity : 0) + (a->slot_mapping ? a->slot_capacity : 0));
  if (a->slot_mapping && (reinterpret_cast<uintptr_t>(a->slot_mapping) & (a->slot_is_int64 ? 7u : 3u)))
    return fail(YL_ERR_ALIGNMENT, "yl_build_index: slot_mapping is not aligned to its element size");

  p.prior_len = a->prior_len;
  p.new_len = a->new_len;
  p.page_table = a->page_table;
  p.table_index = a->table_index;
  p.page_table_stride = a->page_table_stride;
  p.num_pages = a->num_pages;
  p.indices_cap = a->kv_indices ? a->kv_indices_capacity : 0;
  p.slots_cap = a->slot_mapping ? a->slot_capacity : 0;
  p.kv_indptr = a->kv_indptr;
  p.kv_indices = a->kv_indices;
  p.last_page_len = a->kv_last_page_len;
  p.qo_indptr = a->qo_indptr;
  p.slot_mapping = a->slot_mapping;
  p.error_word = a->error_word;
  p.num_table_rows = a->num_table_rows;
  p.max_pages_per_row = a->max_pages_per_row;
  p.page_size = a->page_size;
  p.batch = a->batch_size;
  p.slot64 = a->slot_is_int64;
  p.by_page = FastDiv(static_cast<uint32_t>(a->page_size));
  p.expected_tokens = -1;
  p.beside_store = 0;

  return YL_OK;
}

int launch_index(const IndexParams &p, cudaStream_t stream) {
  // Blocks: one fill element per thread; each block scans the whole batch,
  // so big batches use 1024-thread blocks (4x fewer scans), at most one per SM.
  const int64_t work = p.indices_cap + p.slots_cap;
  const int64_t sms = sm_count();
  // A fill of more than two elements per thread of a full 256-thread grid
  // (long contexts: Qwen2-72B decode, 512 sequences of ~1,000 pages) takes the
  // big-batch kernels too, whose fill keeps several page-table loads in flight
  // per thread instead of one.
  const bool heavy = p.batch > kBigBatch || work > 2 * 4 * sms * kIndexThreads;
  // beside a store (a decode step whose store computes its own slots): the
  // 256-thread kernel at two blocks per SM at most, so two of the store's
  // CTAs fit beside them, with the big-batch staging and fill
  const bool big = heavy && !p.beside_store;
  const bool big_narrow = heavy && p.beside_store;
  const int threads = big ? kIndexThreadsBig : kIndexThreads;
  // (beside the store: one block per SM above 1,024 sequences, measured 0.5 us
  // faster at 2,048; two up to 1,024, where one block per SM measured 0.4-2 us slower)
  const int64_t cap = big ? sms : (p.beside_store ? (p.batch > 1024 ? 1 : 2) : 4) * sms;
  int64_t blocks = (work + threads - 1) / threads;
  if (blocks < 1) blocks = 1;
  if (blocks > cap) blocks = cap;

  // Beside a long store (p.beside_store == 2) one block per SM: the store
  // hides the index build's latency, and fewer index blocks keep fewer of the
  // store's CTAs waiting for room (decode B = 256, 67 MB store: 13.57 ->
  // 13.35 us; Qwen2-72B decode, 336 MB: 61.4 -> 60.0 us).  Beside a short
  // store the index build's latency sets the step and two per SM stay
  // (Qwen2-72B at one head per GPU, 42 MB: 14.0 us, 14.6 at one per SM).
  bool narrow = big_narrow;
  if (p.beside_store == 2 && blocks > sms) {
    blocks = sms;
    narrow = true;
  }
  if (p.batch <= kSmemBatchLimit) {
    const int rc = ensure_smem_attr();
    if (rc != YL_OK) return rc;
    using IndexKernel = void (*)(IndexParams);
    const IndexKernel fn = big ? build_index_kernel<kIndexThreadsBig>
                               : (narrow ? build_index_kernel<kIndexThreads, true> : build_index_kernel<kIndexThreads>);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(blocks));
    cfg.blockDim = dim3(big ? kIndexThreadsBig : kIndexThreads);
    cfg.dynamicSmemBytes = single_launch_smem(p.batch);
    cfg.stream = stream;
    // A programmatic dependent of the kernel before it in the stream: its
    // blocks are placed while that kernel drains and wait (griddepcontrol)
    // for it to complete before reading anything, which hides the launch
    // latency (decode step, 256 sequences: 13.89 -> 13.57 us).
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t err = cudaLaunchKernelEx(&cfg, fn, p);
    if (err != cudaSuccess) {
      cudaGetLastError();
      set_last_error(std::string("yl_build_index launch: ") + cudaGetErrorString(err));
      return YL_ERR_CUDA;
    }
    return check_launch("yl_build_index launch");
  }
  scan_index_kernel<<<1, kScanThreads, 0, stream>>>(p);
  int rc = check_launch("yl_build_index scan launch");
  if (rc != YL_OK) return rc;
  fill_index_kernel<<<static_cast<unsigned>(blocks), kIndexThreadsBig, 0, stream>>>(p);
  return check_launch("yl_build_index fill launch");
}

}  // namespace ylk

extern "C" int yl_build_index(const yl_index_args *a, cudaStream_t stream) {
  using namespace ylk;
  clear_last_error();
  IndexParams p;
  const int rc = prepare_index(a, p);
  if (rc != YL_OK) return rc;
  return launch_index(p, stream);
}
