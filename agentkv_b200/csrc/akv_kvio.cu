// akv_kvio.cu — a model layer's KV in and out of the pool.
//
// The reference's HuggingFace cache (agentkv/hf_cache.py:100-153) writes each
// new token's K and V rows into the pool one token at a time
// (`_kv_data[block, layer, 0/1, :, slot, :] = states[0, :, i, :]`) and then
// rebuilds the layer's whole K and V as contiguous [heads, tokens, head_dim]
// tensors by advanced indexing plus a permute (`_kv_data[block_ids, layer]`,
// `.permute(1, 0, 2, 3).reshape(...)`, truncated to the sequence length).
// Here each is one launch:
//   k_kv_scatter — rows of the new tokens (any head/token strides of the
//                  source, head_dim contiguous) into their (block, slot);
//   k_kv_gather  — for every (K/V, head, block of the table) the block's
//                  [bs, head_dim] tile of this layer, which is contiguous in
//                  the pool, to its place in the contiguous output (the last
//                  block's tile cut to the sequence length).  When every
//                  address and the row size are 16-byte multiples
//                  (the usual case) each tile moves as one bulk copy through
//                  shared memory (k_kv_gather_bulk), else with vector loads
//                  and stores of the widest word that fits.
// Both move bits only; pool block b is the span [b * bpb, (b + 1) * bpb) laid
// out [L][2][H][bs][head_dim].
#include "akv_bulk.cuh"

namespace {

constexpr int kKvThreads = 128;
constexpr int kKvUnroll = 4;

template <typename W>
__global__ void __launch_bounds__(kKvThreads)
k_kv_gather(const char* __restrict__ pool, int64_t bpb, int32_t total, int32_t H, int32_t bs,
            int64_t row_bytes, int64_t layer_off, const int32_t* __restrict__ block_ids, int32_t n_blocks,
            int64_t n_tokens, char* __restrict__ out_k, char* __restrict__ out_v, AkvStatus* st) {
  if (akv_failed(st)) return;
  const int64_t tile_bytes = static_cast<int64_t>(bs) * row_bytes;
  const int64_t n_tiles = 2ll * H * n_blocks;
  for (int64_t t = blockIdx.x; t < n_tiles; t += gridDim.x) {
    // tile order: (kv, head, block) with the block fastest, so consecutive
    // CTAs write consecutive stretches of the output
    const int32_t j = static_cast<int32_t>(t % n_blocks);
    const int64_t kh = t / n_blocks;
    const int32_t h = static_cast<int32_t>(kh % H);
    const int32_t kv = static_cast<int32_t>(kh / H);
    const int32_t b = block_ids[j];
    if (static_cast<uint32_t>(b) >= static_cast<uint32_t>(total)) {
      if (kv == 0 && h == 0 && threadIdx.x == 0) akv_fail(st, AKV_ERR_OUT_OF_RANGE, j, b, total);
      continue;
    }
    const int64_t first = static_cast<int64_t>(j) * bs;
    const int64_t rows = min(static_cast<int64_t>(bs), n_tokens - first);
    if (rows <= 0) continue;  // a block past the sequence end
    const W* __restrict__ src = reinterpret_cast<const W*>(
        pool + static_cast<int64_t>(b) * bpb + layer_off + (static_cast<int64_t>(kv) * H + h) * tile_bytes);
    W* __restrict__ dst = reinterpret_cast<W*>((kv ? out_v : out_k) +
                                               (static_cast<int64_t>(h) * n_tokens + first) * row_bytes);
    const int64_t words = rows * row_bytes / static_cast<int64_t>(sizeof(W));
    // all of a thread's loads of a pass are issued before its stores, so a
    // 4 KiB tile is one round trip to HBM
    for (int64_t base = threadIdx.x; base < words; base += kKvThreads * kKvUnroll) {
      W r[kKvUnroll];
#pragma unroll
      for (int u = 0; u < kKvUnroll; ++u) {
        const int64_t w = base + static_cast<int64_t>(u) * kKvThreads;
        if (w < words) r[u] = src[w];
      }
#pragma unroll
      for (int u = 0; u < kKvUnroll; ++u) {
        const int64_t w = base + static_cast<int64_t>(u) * kKvThreads;
        if (w < words) dst[w] = r[u];
      }
    }
  }
}

// Bulk-copy gather: one warp per CTA, several CTAs per SM.  The warp works
// out 32 tiles' addresses at a time (lane i: its tile's block id, source,
// destination and byte count), and lane 0 moves them with bulk copies —
// global -> shared on an mbarrier, then shared -> global — kStages tiles in
// flight.  Tiles are dealt to the CTAs round robin (tile t to CTA t mod
// grid).  Every wait is bounded; a timeout sets AKV_ERR_TIMEOUT, lets the
// loads in flight land and returns.
template <int kStages>
__global__ void __launch_bounds__(32)
k_kv_gather_bulk(const char* __restrict__ pool, int64_t bpb, int32_t total, int32_t H, int32_t bs,
                 int64_t row_bytes, int64_t layer_off, const int32_t* __restrict__ block_ids, int32_t n_blocks,
                 int64_t n_tokens, char* __restrict__ out_k, char* __restrict__ out_v, AkvStatus* st) {
  constexpr uint32_t kFull = 0xffffffffu;
  extern __shared__ __align__(1024) unsigned char smem[];
  __shared__ __align__(8) uint64_t bars[kStages];
  __shared__ char* dsts[kStages];
  __shared__ uint32_t sizes[kStages];
  const int lane = threadIdx.x;
  if (akv_failed(st)) return;
  const int64_t tile = static_cast<int64_t>(bs) * row_bytes;
  if (lane == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(smem_u32(&bars[s]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
  const int64_t n_items = 2ll * H * n_blocks;
  const int64_t grid = gridDim.x;
  int64_t next_group = 0;  // this CTA's k-th tiles are blockIdx.x + k * grid
  const char* my_src = nullptr;
  char* my_dst = nullptr;
  uint32_t my_bytes = 0;
  int cur = 32;  // position in the current group of 32 (32: take the next group)
  bool more = true;
  auto load_group = [&]() {
    const int64_t t = blockIdx.x + (next_group * 32 + lane) * grid;
    ++next_group;
    my_bytes = 0;
    if (t < n_items) {
      const int32_t j = static_cast<int32_t>(t % n_blocks);
      const int64_t kh = t / n_blocks;
      const int32_t h = static_cast<int32_t>(kh % H);
      const int32_t kv = static_cast<int32_t>(kh / H);
      const int32_t b = block_ids[j];
      const int64_t first = static_cast<int64_t>(j) * bs;
      const int64_t rows = min(static_cast<int64_t>(bs), n_tokens - first);
      if (static_cast<uint32_t>(b) >= static_cast<uint32_t>(total)) {
        if (kv == 0 && h == 0) akv_fail(st, AKV_ERR_OUT_OF_RANGE, j, b, total);
      } else if (rows > 0) {
        my_src = pool + static_cast<int64_t>(b) * bpb + layer_off + (static_cast<int64_t>(kv) * H + h) * tile;
        my_dst = (kv ? out_v : out_k) + (static_cast<int64_t>(h) * n_tokens + first) * row_bytes;
        my_bytes = static_cast<uint32_t>(rows * row_bytes);
      }
    }
    // any lane past the end means later groups are empty too
    more = __ballot_sync(kFull, t < n_items) == kFull;
  };
  // The next tile to move (warp-uniform); false when there is none.
  auto next_tile = [&](const char*& src, char*& dst, uint32_t& bytes) -> bool {
    while (true) {
      if (cur == 32) {
        if (next_group > 0 && !more) return false;
        load_group();
        cur = 0;
      }
      const uint32_t has = __ballot_sync(kFull, my_bytes != 0) & (kFull << cur);
      if (!has) {
        cur = 32;
        continue;
      }
      const int l = __ffs(has) - 1;
      src = reinterpret_cast<const char*>(__shfl_sync(kFull, reinterpret_cast<uint64_t>(my_src), l));
      dst = reinterpret_cast<char*>(__shfl_sync(kFull, reinterpret_cast<uint64_t>(my_dst), l));
      bytes = __shfl_sync(kFull, my_bytes, l);
      cur = l + 1;
      return true;
    }
  };
  auto issue = [&](int64_t m, const char* src, char* dst, uint32_t bytes) {
    if (lane == 0) {
      const int s = static_cast<int>(m % kStages);
      dsts[s] = dst;
      sizes[s] = bytes;
      const uint32_t bar = smem_u32(&bars[s]);
      mbar_expect_tx(bar, bytes);
      bulk_load(smem_u32(smem + static_cast<size_t>(s) * tile), src, bytes, bar);
    }
  };
  int64_t loads = 0, stores = 0;
  const char* src;
  char* dst;
  uint32_t bytes;
  while (loads < kStages && next_tile(src, dst, bytes)) issue(loads++, src, dst, bytes);
  bool timed_out = false;
  while (stores < loads) {
    const int s = static_cast<int>(stores % kStages);
    const uint32_t parity = static_cast<uint32_t>((stores / kStages) & 1);
    int ok = 1;
    if (lane == 0) {
      ok = mbar_wait(smem_u32(&bars[s]), parity) ? 1 : 0;
      if (ok) {
        bulk_store(dsts[s], smem_u32(smem + static_cast<size_t>(s) * tile), sizes[s]);
        bulk_commit();
      } else {
        akv_fail(st, AKV_ERR_TIMEOUT, static_cast<int32_t>(blockIdx.x), -1, 0, stores);
      }
    }
    if (!__shfl_sync(kFull, ok, 0)) {
      timed_out = true;
      break;
    }
    ++stores;
    // the store issued one iteration ago has finished reading its stage
    if (stores >= 2) {
      if (lane == 0) bulk_wait_read<1>();
      __syncwarp();
      if (next_tile(src, dst, bytes)) issue(loads++, src, dst, bytes);
    }
  }
  if (lane == 0) {
    if (timed_out) {
      for (int64_t m = stores + 1; m < loads; ++m)
        mbar_wait(smem_u32(&bars[m % kStages]), static_cast<uint32_t>((m / kStages) & 1));
    }
    // The CTA may leave once its stores have read their shared-memory
    // stages; their writes complete with the grid (waiting for them here
    // only lengthens the kernel's tail).
    bulk_wait_read<0>();
  }
}

constexpr int kGatherStages = 8;
constexpr int kGatherCtasPerSm = 4;
constexpr int64_t kGatherMaxTile = 16 * 1024;  // stage size limit: 8 x 16 KiB per CTA

template <typename W>
__global__ void __launch_bounds__(kKvThreads)
k_kv_scatter(char* __restrict__ pool, int64_t bpb, int32_t total, int32_t H, int32_t bs, int64_t row_bytes,
             int64_t layer_off, const int32_t* __restrict__ slots, int32_t n_new,
             const char* __restrict__ k_src, const char* __restrict__ v_src, int64_t stride_h,
             int64_t stride_t, AkvStatus* st) {
  if (akv_failed(st)) return;
  const int64_t words_per_row = row_bytes / static_cast<int64_t>(sizeof(W));
  const int64_t n_rows = 2ll * H * n_new;
  const int64_t n_words = n_rows * words_per_row;
  for (int64_t x = blockIdx.x * static_cast<int64_t>(kKvThreads) + threadIdx.x; x < n_words;
       x += static_cast<int64_t>(gridDim.x) * kKvThreads) {
    const int64_t r = x / words_per_row;
    const int64_t w = x - r * words_per_row;
    const int32_t i = static_cast<int32_t>(r % n_new);  // token
    const int64_t kh = r / n_new;
    const int32_t h = static_cast<int32_t>(kh % H);
    const int32_t kv = static_cast<int32_t>(kh / H);
    const int32_t slot = slots[i];
    const int32_t b = slot / bs;
    if (slot < 0 || static_cast<uint32_t>(b) >= static_cast<uint32_t>(total)) {
      if (w == 0 && kv == 0 && h == 0) akv_fail(st, AKV_ERR_OUT_OF_RANGE, i, slot, total);
      continue;
    }
    const int32_t pos = slot - b * bs;
    const W* src = reinterpret_cast<const W*>((kv ? v_src : k_src) + h * stride_h + i * stride_t);
    W* dst = reinterpret_cast<W*>(pool + static_cast<int64_t>(b) * bpb + layer_off +
                                  ((static_cast<int64_t>(kv) * H + h) * bs + pos) * row_bytes);
    dst[w] = src[w];
  }
}

// Widest word (16, 8, 4, 2 or 1 bytes) dividing every address and size.
int kv_word(uint64_t bits) {
  for (int w = 16; w > 1; w >>= 1)
    if ((bits & static_cast<uint64_t>(w - 1)) == 0) return w;
  return 1;
}

int kv_grid(int64_t work) {
  const int64_t cap = static_cast<int64_t>(kAkvSMs) * 16;
  return static_cast<int>(work < 1 ? 1 : (work < cap ? work : cap));
}

}  // namespace

int akv_kvio_prepare() {
#define AKV_LOAD(fn) if (int rc = akv_load_kernel(reinterpret_cast<const void*>(fn), "akv_prepare: " #fn)) return rc
  AKV_LOAD(k_kv_gather_bulk<kGatherStages>);
  if (cudaFuncSetAttribute(reinterpret_cast<const void*>(k_kv_gather_bulk<kGatherStages>),
                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(kGatherStages * kGatherMaxTile)) != cudaSuccess)
    return akv_cuda_fail(cudaGetLastError(), "akv_prepare: k_kv_gather_bulk shared memory");
  AKV_LOAD(k_kv_gather<uint4>);
  AKV_LOAD(k_kv_gather<uint2>);
  AKV_LOAD(k_kv_gather<uint32_t>);
  AKV_LOAD(k_kv_gather<uint16_t>);
  AKV_LOAD(k_kv_gather<uint8_t>);
  AKV_LOAD(k_kv_scatter<uint4>);
  AKV_LOAD(k_kv_scatter<uint2>);
  AKV_LOAD(k_kv_scatter<uint32_t>);
  AKV_LOAD(k_kv_scatter<uint16_t>);
  AKV_LOAD(k_kv_scatter<uint8_t>);
#undef AKV_LOAD
  return AKV_OK;
}

extern "C" int akv_kv_gather(const void* pool, int32_t total_blocks, int32_t num_layers, int32_t num_kv_heads,
                             int32_t block_size, int64_t row_bytes, int32_t layer, const int32_t* block_ids,
                             int32_t n_blocks, int64_t n_tokens, void* out_k, void* out_v, AkvStatus* status,
                             void* stream) {
  AKV_ARG_CHECK(pool && out_k && out_v && (block_ids || n_blocks == 0), "akv_kv_gather: NULL pointer");
  AKV_ARG_CHECK(total_blocks > 0 && num_layers > 0 && num_kv_heads > 0 && block_size > 0 && row_bytes > 0,
                "akv_kv_gather: bad geometry");
  AKV_ARG_CHECK(layer >= 0 && layer < num_layers, "akv_kv_gather: layer %d of %d", layer, num_layers);
  AKV_ARG_CHECK(n_blocks >= 0 && n_tokens >= 0 && n_tokens <= static_cast<int64_t>(n_blocks) * block_size,
                "akv_kv_gather: %lld tokens exceed %d blocks of %d", static_cast<long long>(n_tokens), n_blocks,
                block_size);
  if (n_tokens == 0) return AKV_OK;
  const int64_t tile = static_cast<int64_t>(block_size) * row_bytes;
  const int64_t bpb = static_cast<int64_t>(num_layers) * 2 * num_kv_heads * tile;
  const int64_t layer_off = static_cast<int64_t>(layer) * 2 * num_kv_heads * tile;
  const uint64_t bits = reinterpret_cast<uintptr_t>(pool) | reinterpret_cast<uintptr_t>(out_k) |
                        reinterpret_cast<uintptr_t>(out_v) | static_cast<uint64_t>(row_bytes);
  const int w = kv_word(bits);
  cudaStream_t s = akv_stream(stream);
  if (w == 16 && tile <= kGatherMaxTile) {
    const int64_t tiles = 2ll * num_kv_heads * n_blocks;
    const int64_t cap = static_cast<int64_t>(kAkvSMs) * kGatherCtasPerSm;
    const int grid_b = static_cast<int>(tiles < cap ? tiles : cap);
    k_kv_gather_bulk<kGatherStages><<<grid_b, 32, static_cast<size_t>(kGatherStages * tile), s>>>(
        static_cast<const char*>(pool), bpb, total_blocks, num_kv_heads, block_size, row_bytes, layer_off,
        block_ids, n_blocks, n_tokens, static_cast<char*>(out_k), static_cast<char*>(out_v), status);
    AKV_LAUNCH_CHECK("akv_kv_gather(bulk)");
    return AKV_OK;
  }
  const int grid = kv_grid(2ll * num_kv_heads * n_blocks);
  // (A variant that took 4 tiles per CTA and issued all their loads at once
  // measured slower: 11.9 us against 9.8 us for a 4,096-token layer.)
#define AKV_GATHER(W)                                                                                        \
  k_kv_gather<W><<<grid, kKvThreads, 0, s>>>(static_cast<const char*>(pool), bpb, total_blocks, num_kv_heads, \
                                             block_size, row_bytes, layer_off, block_ids, n_blocks, n_tokens, \
                                             static_cast<char*>(out_k), static_cast<char*>(out_v), status)
  switch (w) {
    case 16: AKV_GATHER(uint4); break;
    case 8: AKV_GATHER(uint2); break;
    case 4: AKV_GATHER(uint32_t); break;
    case 2: AKV_GATHER(uint16_t); break;
    default: AKV_GATHER(uint8_t); break;
  }
#undef AKV_GATHER
  AKV_LAUNCH_CHECK("akv_kv_gather");
  return AKV_OK;
}

extern "C" int akv_kv_scatter(void* pool, int32_t total_blocks, int32_t num_layers, int32_t num_kv_heads,
                              int32_t block_size, int64_t row_bytes, int32_t layer, const int32_t* slots,
                              int32_t n_new, const void* k_src, const void* v_src, int64_t src_stride_head,
                              int64_t src_stride_token, AkvStatus* status, void* stream) {
  AKV_ARG_CHECK(n_new >= 0, "akv_kv_scatter: n_new=%d", n_new);
  if (n_new == 0) return AKV_OK;
  AKV_ARG_CHECK(pool && slots && k_src && v_src, "akv_kv_scatter: NULL pointer");
  AKV_ARG_CHECK(total_blocks > 0 && num_layers > 0 && num_kv_heads > 0 && block_size > 0 && row_bytes > 0,
                "akv_kv_scatter: bad geometry");
  AKV_ARG_CHECK(layer >= 0 && layer < num_layers, "akv_kv_scatter: layer %d of %d", layer, num_layers);
  AKV_ARG_CHECK(src_stride_head >= 0 && src_stride_token >= 0, "akv_kv_scatter: negative stride");
  const int64_t tile = static_cast<int64_t>(block_size) * row_bytes;
  const int64_t bpb = static_cast<int64_t>(num_layers) * 2 * num_kv_heads * tile;
  const int64_t layer_off = static_cast<int64_t>(layer) * 2 * num_kv_heads * tile;
  const uint64_t bits = reinterpret_cast<uintptr_t>(pool) | reinterpret_cast<uintptr_t>(k_src) |
                        reinterpret_cast<uintptr_t>(v_src) | static_cast<uint64_t>(row_bytes) |
                        static_cast<uint64_t>(src_stride_head) | static_cast<uint64_t>(src_stride_token);
  const int w = kv_word(bits);
  const int64_t words = 2ll * num_kv_heads * n_new * (row_bytes / w);
  const int grid = kv_grid((words + kKvThreads - 1) / kKvThreads);
  cudaStream_t s = akv_stream(stream);
#define AKV_SCATTER(W)                                                                                        \
  k_kv_scatter<W><<<grid, kKvThreads, 0, s>>>(static_cast<char*>(pool), bpb, total_blocks, num_kv_heads,       \
                                              block_size, row_bytes, layer_off, slots, n_new,                  \
                                              static_cast<const char*>(k_src), static_cast<const char*>(v_src), \
                                              src_stride_head, src_stride_token, status)
  switch (w) {
    case 16: AKV_SCATTER(uint4); break;
    case 8: AKV_SCATTER(uint2); break;
    case 4: AKV_SCATTER(uint32_t); break;
    case 2: AKV_SCATTER(uint16_t); break;
    default: AKV_SCATTER(uint8_t); break;
  }
#undef AKV_SCATTER
  AKV_LAUNCH_CHECK("akv_kv_scatter");
  return AKV_OK;
}
