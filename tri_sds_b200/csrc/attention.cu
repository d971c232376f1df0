// Verify / decode attention over the KV cache (GQA), head_dim 128.
//
// Work unit = (sequence b, kv head, key split).  The R = T * (Hq/Hkv) query
// rows that share a kv head (T new tokens x the q heads of the group) are
// processed together, so every K/V byte is read from HBM once per step
// (the reference's GQA kernel re-reads K/V once per q head,
// attention.py:237-296; its verify path materialises repeat_interleave
// copies, qwen_model.py:122-123).
//
// * K/V tiles of 64 keys x 128 dims are staged by TMA (cp.async.bulk.tensor,
//   128-byte swizzle, two 64-column boxes per tile) into a STAGES-deep
//   shared-memory ring, completion tracked by mbarriers (bounded waits).
// * Each warp owns 16 query rows.  S = Q K^T and O += P V run on the
//   tensor cores (mma.m16n8k16 bf16 -> fp32); Q fragments stay in
//   registers; K / V fragments come from the swizzled tiles by ldmatrix.
// * fp32 online softmax in the exp2 domain; row max / sum across the four
//   lanes sharing a row by shuffles.
// * Keys are split into fixed chunks of `split_keys` rows, and a split's
//   tiles into KG key groups (a function of split_keys alone).  With one
//   split the rows are normalised in place; otherwise a split writes its
//   unnormalised O with (m, l) to the workspace and a combine pass merges
//   the splits in index order.  Split and key-group boundaries depend only
//   on the key index, and masked / empty splits contribute exact zeros, so a
//   query's output is bit-identical whether it is verified with T tokens or
//   decoded alone.
// * The K/V cache is contiguous ([B][Hkv][S][D], tsds_verify_attention) or
//   paged in token pools through a request-to-token table
//   (tsds_verify_attention_paged); both feed the same consumers.
#include "common.cuh"
#include "linear.cuh"
#include "tc_core.cuh"

using namespace tsds;

namespace {

constexpr int D = 128;
constexpr int TILE = 64;                    // keys per tile
constexpr int ATT_MAX_WARPS = 8;            // consumer warps per CTA (row groups x key groups)
constexpr int ATT_STAGES = 6;               // K/V tiles in flight per CTA
// Ring invariant: a consumer's next tile is KG tiles after its last one, and
// it waits for that tile's full barrier by phase parity.  The wait is exact
// only if the tile STAGES before it - the stage's previous use - has landed;
// with KG dividing STAGES that tile belongs to the same key group, so the
// waiting warp has already consumed it.  Every KG below divides ATT_STAGES.
constexpr int HALF_BYTES = TILE * 128;      // one 64x64 bf16 box = 8 KB
constexpr int TILE_BYTES = 4 * HALF_BYTES;  // K lo/hi + V lo/hi = 32 KB
constexpr float LOG2E = 1.4426950408889634f;

__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// Byte offset of (key, 16-byte chunk c16 in [0,16)) inside a K or V tile
// stored as two swizzled 64-column halves (TMA SWIZZLE_128B pattern:
// chunk index XOR (row & 7) within each 128-byte row).
__device__ __forceinline__ uint32_t tile_off(int key, int c16) {
  const int half = c16 >> 3, c = c16 & 7;
  return half * HALF_BYTES + key * 128 + ((c ^ (key & 7)) << 4);
}

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

struct AttnArgs {
  const bf16* q;
  bf16* out;
  const int32_t* starts;
  const uint32_t* tree_mask;
  float* ws_o;    // [B*Hkv][nsplit][Rpad][D]
  float2* ws_ml;  // [B*Hkv][nsplit][Rpad]
  int32_t* status;
  int B, T, Hq, Hkv, S, G, R, Rpad, nsplit, split_keys, nrb, mask_origin;
  float scale_log2;
  int cl;  // tcgen05 variant: the splits of a row block form a cluster and combine through shared memory
  int RG, KG;  // default kernel: 16-row groups per row block, key groups per split
  // Paged KV (default kernel): 0 = contiguous caches [B][Hkv][S][D] through
  // the tensor maps; otherwise K/V live in token pools [pool_rows][Hkv][D]
  // and key p of sequence b is pool row table[req(b) * table_ld + p]
  // (req(b) = req_rows[b], or b without req_rows).  1: every aligned run of
  // 64 keys sits in 64 consecutive pool rows (pages of a multiple of 64
  // tokens), staged by TMA through tensor maps over the pools; 2: rows
  // gathered one by one by the producer warp's 32 lanes (cp.async).
  int paged;
  const bf16* k_pool;
  const bf16* v_pool;
  const int32_t* table;
  const int64_t* req_rows;
  int64_t table_ld, pool_rows;
};

// 16-byte global -> shared copy (L2 only), completion tracked per thread
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

// the calling thread's earlier cp.async copies arrive on the barrier when
// they land (one arrival per thread, counted against the barrier's count)
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// pool row of key `pos` of sequence b (paged KV); a row outside the pool is
// recorded as TSDS_E_INDEX and replaced by row 0 (never read out of range)
__device__ __forceinline__ int64_t kv_slot(const AttnArgs& a, int b, int pos) {
  const int64_t req = a.req_rows ? a.req_rows[b] : b;
  const int64_t slot = a.table[req * a.table_ld + pos];
  if (slot < 0 || slot >= a.pool_rows) {
    atomicExch(a.status, TSDS_E_INDEX);
    return 0;
  }
  return slot;
}

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// named barrier that also ANDs a predicate over its threads: every thread
// gets the same answer
__device__ __forceinline__ bool named_bar_and(int id, int threads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(threads)
      : "memory");
  return r != 0;
}

// Persistent, warp-specialised split-KV attention.  One CTA per SM walks the
// work items (b, kv head, row block, key split) i = blockIdx.x, + gridDim.x,
// ...  Warp 0 (one lane) streams every K/V tile of the CTA's items, item
// after item, through a STAGES-deep ring (full / empty mbarriers), so the
// next item's tiles arrive while the consumers finish the current one.
// Consumer warp c owns 16 query rows (row group c % RG of the item's row
// block) and the split's tiles of key group c / RG (tiles t = kg, kg + KG,
// ... of the split); at the end of an item the KG key groups' (m, l, O) of a
// row are merged in key-group order through shared memory, then the item's
// rows are normalised in place (one split) or written as a split partial.
// KG depends only on split_keys and a tile's key group only on its key
// index, so a row's result never depends on T, on its row block or on the
// grid.
template <int STAGES>
__global__ void __launch_bounds__(32 * (1 + ATT_MAX_WARPS), 1)
    verify_attn_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                       AttnArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the 128B-swizzle atoms; the merge area follows the ring
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* xs = reinterpret_cast<float*>(smem + STAGES * TILE_BYTES);
  __shared__ uint64_t full_bar[STAGES];
  __shared__ uint64_t empty_bar[STAGES];
  __shared__ int s_abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int RG = a.RG, KG = a.KG, NC = a.RG * a.KG;
  const int items_per_b = a.Hkv * a.nrb * a.nsplit;
  const int nitems = a.B * items_per_b;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      // a TMA stage completes on one arrival + its bytes; a gathered stage
      // on the producer warp's 32 cp.async arrivals
      mbar_init(&full_bar[s], a.paged == 2 ? 32 : 1);
      mbar_init(&empty_bar[s], RG);  // the row groups of the tile's key group
    }
    s_abort = 0;
    fence_barrier_init();
  }
  __syncthreads();
  pdl_trigger();
  pdl_wait();

  // item -> (b, kvh, rb, split) and the key range it covers
  struct Item {
    int b, kvh, rb, split, key_begin, ntiles, kv_len;
  };
  auto decode = [&](int item) {
    Item it;
    it.b = item / items_per_b;
    int r = item % items_per_b;
    it.kvh = r / (a.nrb * a.nsplit);
    r %= a.nrb * a.nsplit;
    it.split = r / a.nrb;
    it.rb = r % a.nrb;
    it.kv_len = a.starts[it.b] + a.T;
    it.key_begin = it.split * a.split_keys;
    const int key_end = min(it.key_begin + a.split_keys, it.kv_len);
    it.ntiles = key_end > it.key_begin ? (key_end - it.key_begin + TILE - 1) / TILE : 0;
    return it;
  };

  if (warp == 0) {
    // ---------------- producer ----------------
    if (a.paged == 2) {
      // Gathered rows: lane l copies 16-byte chunk l % 16 of keys 2i + l / 16
      // (i = 0..31) of K and of V, so a warp-wide copy moves two whole
      // 256-byte rows; the chunks land where TMA's 128-byte swizzle would
      // put them.  Keys past the sequence repeat its last row (masked).
      int q = 0;
      bool stop = false;
      const int hw = lane >> 4, c16 = lane & 15;
      for (int item = blockIdx.x; item < nitems && !stop; item += gridDim.x) {
        const Item it = decode(item);
        for (int t = 0; t < it.ntiles; ++t, ++q) {
          const int s = q % STAGES;
          const bool ok = q < STAGES || mbar_wait(&empty_bar[s], ((q / STAGES) - 1) & 1);
          if (!__all_sync(0xffffffffu, ok && !*(volatile int*)&s_abort)) {
            if (lane == 0 && !ok) {
              atomicExch(a.status, TSDS_E_TIMEOUT);
              s_abort = 1;
            }
            stop = true;
            break;
          }
          const int key0 = it.key_begin + t * TILE;
          // lane l looks up keys key0 + l and key0 + 32 + l; the others by shuffle
          const int64_t sl0 = kv_slot(a, it.b, min(key0 + lane, it.kv_len - 1));
          const int64_t sl1 = kv_slot(a, it.b, min(key0 + 32 + lane, it.kv_len - 1));
          const uint32_t stage = smem_u32(smem + s * TILE_BYTES);
#pragma unroll 4
          for (int i = 0; i < 32; ++i) {
            const int key = 2 * i + hw;
            const int64_t slot = __shfl_sync(0xffffffffu, key < 32 ? sl0 : sl1, key & 31);
            const int64_t off = (slot * a.Hkv + it.kvh) * D + c16 * 8;
            const uint32_t d = stage + tile_off(key, c16);
            cp_async16(d, a.k_pool + off);
            cp_async16(d + 2 * HALF_BYTES, a.v_pool + off);
          }
          cp_async_arrive(&full_bar[s]);
        }
      }
      // every lane's copies land before the CTA can exit
      drain_tma_ring(full_bar, STAGES, q);
      return;
    }
    if (lane == 0) {
      prefetch_tmap(&kmap);
      prefetch_tmap(&vmap);
      int q = 0;  // ring sequence number of the next tile
      bool stop = false;
      // The first tile of a first split is needed whatever the sequence's
      // length (it holds at least one key): with the contiguous cache its
      // rows are known from the indices alone, so it is requested before
      // the sequence lengths are read.
      bool first_early = false;
      if (!a.paged && (int)blockIdx.x < nitems) {
        const int item = blockIdx.x, b0 = item / items_per_b, r0 = item % items_per_b;
        const int kvh0 = r0 / (a.nrb * a.nsplit), split0 = (r0 % (a.nrb * a.nsplit)) / a.nrb;
        if (split0 == 0) {
          const int row = (int)(((int64_t)b0 * a.Hkv + kvh0) * a.S);
          mbar_arrive_expect_tx(&full_bar[0], TILE_BYTES);
          tma_load_2d(smem + 0 * HALF_BYTES, &kmap, &full_bar[0], 0, row);
          tma_load_2d(smem + 1 * HALF_BYTES, &kmap, &full_bar[0], 64, row);
          tma_load_2d(smem + 2 * HALF_BYTES, &vmap, &full_bar[0], 0, row);
          tma_load_2d(smem + 3 * HALF_BYTES, &vmap, &full_bar[0], 64, row);
          first_early = true;
        }
      }
      for (int item = blockIdx.x; item < nitems && !stop; item += gridDim.x) {
        const Item it = decode(item);
        const int ntiles = it.ntiles, key_begin = it.key_begin;
        const int64_t slab_row = ((int64_t)it.b * a.Hkv + it.kvh) * a.S;
        for (int t = 0; t < ntiles; ++t, ++q) {
          if (q == 0 && first_early) continue;  // requested above
          const int s = q % STAGES;
          if (q >= STAGES && !mbar_wait(&empty_bar[s], ((q / STAGES) - 1) & 1)) {
            atomicExch(a.status, TSDS_E_TIMEOUT);
            s_abort = 1;
            stop = true;
            break;
          }
          if (*(volatile int*)&s_abort) {
            stop = true;
            break;
          }
          uint8_t* dst = smem + s * TILE_BYTES;
          // contiguous: the slab's rows; paged (64-key pages): the page's
          // first pool row, the kv head's 128 columns of the pool row
          const int row = a.paged ? (int)kv_slot(a, it.b, key_begin + t * TILE) : (int)(slab_row + key_begin + t * TILE);
          const int col = a.paged ? it.kvh * D : 0;
          mbar_arrive_expect_tx(&full_bar[s], TILE_BYTES);
          tma_load_2d(dst + 0 * HALF_BYTES, &kmap, &full_bar[s], col, row);
          tma_load_2d(dst + 1 * HALF_BYTES, &kmap, &full_bar[s], col + 64, row);
          tma_load_2d(dst + 2 * HALF_BYTES, &vmap, &full_bar[s], col, row);
          tma_load_2d(dst + 3 * HALF_BYTES, &vmap, &full_bar[s], col + 64, row);
        }
      }
      // every requested tile lands before the CTA can exit
      drain_tma_ring(full_bar, STAGES, q);
    }
    return;
  }

  // ---------------- consumers ----------------
  const int cw = warp - 1, rg = cw % RG, kg = cw / RG;
  const int g = lane >> 2, tig = lane & 3;
  const uint32_t smem_base = smem_u32(smem);
  int q0 = 0;  // ring sequence number of the current item's first tile
  for (int item = blockIdx.x; item < nitems; item += gridDim.x) {
    const Item it = decode(item);
    // a split past the end of its sequence holds no keys: the combine pass
    // reads only splits below the sequence's length, so it is skipped whole
    // (every consumer warp takes the same decision; the producer streams no
    // tiles for it)
    if (it.ntiles == 0) continue;
    const int b = it.b, kvh = it.kvh, rb = it.rb, split = it.split;
    const int key_begin = it.key_begin, ntiles = it.ntiles, kv_len = it.kv_len;
    const int start = a.starts[b];
    const int64_t unit = ((int64_t)b * a.Hkv + kvh) * a.nsplit + split;
    const int r0 = rb * RG * 16 + rg * 16 + g, r1 = r0 + 8;
    const int t0 = r0 / a.G, t1 = r1 / a.G;
    const bool v0 = r0 < a.R, v1 = r1 < a.R;
    uint32_t qa[8][4];
    {
      const bf16* qp0 = a.q + (((int64_t)b * a.T + (v0 ? t0 : 0)) * a.Hq + kvh * a.G + (v0 ? r0 % a.G : 0)) * D;
      const bf16* qp1 = a.q + (((int64_t)b * a.T + (v1 ? t1 : 0)) * a.Hq + kvh * a.G + (v1 ? r1 % a.G : 0)) * D;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int c = kk * 16 + 2 * tig;
        qa[kk][0] = v0 ? *reinterpret_cast<const uint32_t*>(qp0 + c) : 0u;
        qa[kk][1] = v1 ? *reinterpret_cast<const uint32_t*>(qp1 + c) : 0u;
        qa[kk][2] = v0 ? *reinterpret_cast<const uint32_t*>(qp0 + c + 8) : 0u;
        qa[kk][3] = v1 ? *reinterpret_cast<const uint32_t*>(qp1 + c + 8) : 0u;
      }
    }
    const int mask_base = a.mask_origin >= 0 ? a.mask_origin : start;
    const int ctx_end = min(a.tree_mask ? mask_base : start, kv_len);
    const uint32_t mask0 = (a.tree_mask && v0) ? a.tree_mask[b * a.T + t0] : 0u;
    const uint32_t mask1 = (a.tree_mask && v1) ? a.tree_mask[b * a.T + t1] : 0u;
    const bool tree = a.tree_mask != nullptr;

    float o[16][4];
#pragma unroll
    for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

    for (int tile = kg; tile < ntiles; tile += KG) {
      const int qs = q0 + tile, s = qs % STAGES;
      const int ok = (!*(volatile int*)&s_abort && mbar_wait(&full_bar[s], (qs / STAGES) & 1)) ? 1 : 0;
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) {
          atomicExch(a.status, TSDS_E_TIMEOUT);
          s_abort = 1;
        }
        break;
      }
      const uint32_t kbase = smem_base + s * TILE_BYTES;
      const uint32_t vbase = kbase + 2 * HALF_BYTES;
      const int key0 = key_begin + tile * TILE;

      // S = Q K^T for 64 keys: 8 n-tiles of 8 keys.
      float sc[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 8; kk += 2) {
          const int mi = lane >> 3, ri = lane & 7;
          const int key = j * 8 + ri;
          uint32_t b0, b1, b2, b3;
          ldsm_x4(kbase + tile_off(key, 2 * kk + mi), b0, b1, b2, b3);
          mma_bf16(sc[j], qa[kk], b0, b1);
          mma_bf16(sc[j], qa[kk + 1], b2, b3);
        }
      }
      // mask + row max.  A tile wholly below ctx_end (shared context: keys
      // below the tree's first key or the new tokens, and below kv_len) is
      // visible to every valid row, so it skips the per-key tests.
      float mx0 = -INFINITY, mx1 = -INFINITY;
      if (key0 + TILE <= ctx_end) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            sc[j][e] = v0 ? sc[j][e] * a.scale_log2 : -INFINITY;
            sc[j][2 + e] = v1 ? sc[j][2 + e] * a.scale_log2 : -INFINITY;
            mx0 = fmaxf(mx0, sc[j][e]);
            mx1 = fmaxf(mx1, sc[j][2 + e]);
          }
        }
      } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int kabs = key0 + j * 8 + 2 * tig + e;
          bool vis0 = v0 && kabs < kv_len, vis1 = v1 && kabs < kv_len;
          if (tree) {
            // bit i of a row's mask covers key mask_base + i; keys below are shared context
            const int rel = kabs - mask_base;
            if (rel >= 0) {
              const bool in = rel < 32;
              vis0 = vis0 && in && ((mask0 >> (rel & 31)) & 1u);
              vis1 = vis1 && in && ((mask1 >> (rel & 31)) & 1u);
            }
          } else {
            const int rel = kabs - start;
            vis0 = vis0 && rel <= t0;
            vis1 = vis1 && rel <= t1;
          }
          sc[j][e] = vis0 ? sc[j][e] * a.scale_log2 : -INFINITY;
          sc[j][2 + e] = vis1 ? sc[j][2 + e] * a.scale_log2 : -INFINITY;
          mx0 = fmaxf(mx0, sc[j][e]);
          mx1 = fmaxf(mx1, sc[j][2 + e]);
        }
      }
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      // rows with nothing visible so far keep m = -inf and p = 0
      const float al0 = mn0 == -INFINITY ? 1.f : exp2f(m0 - mn0);
      const float al1 = mn1 == -INFINITY ? 1.f : exp2f(m1 - mn1);
      const float sub0 = mn0 == -INFINITY ? 0.f : mn0;
      const float sub1 = mn1 == -INFINITY ? 0.f : mn1;
      m0 = mn0;
      m1 = mn1;
      float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        sc[j][0] = exp2f(sc[j][0] - sub0);
        sc[j][1] = exp2f(sc[j][1] - sub0);
        sc[j][2] = exp2f(sc[j][2] - sub1);
        sc[j][3] = exp2f(sc[j][3] - sub1);
        ps0 += sc[j][0] + sc[j][1];
        ps1 += sc[j][2] + sc[j][3];
      }
      l0 = l0 * al0 + ps0;
      l1 = l1 * al1 + ps1;
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        o[n][0] *= al0;
        o[n][1] *= al0;
        o[n][2] *= al1;
        o[n][3] *= al1;
      }
      // O += P V: 4 k-steps of 16 keys, 16 n-tiles of 8 dims.
#pragma unroll
      for (int kq = 0; kq < 4; ++kq) {
        uint32_t pa[4];
        pa[0] = pack2(sc[2 * kq][0], sc[2 * kq][1]);
        pa[1] = pack2(sc[2 * kq][2], sc[2 * kq][3]);
        pa[2] = pack2(sc[2 * kq + 1][0], sc[2 * kq + 1][1]);
        pa[3] = pack2(sc[2 * kq + 1][2], sc[2 * kq + 1][3]);
#pragma unroll
        for (int n = 0; n < 16; n += 2) {
          const int mi = lane >> 3, ri = lane & 7;
          const int key = kq * 16 + (mi & 1) * 8 + ri;
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(vbase + tile_off(key, n + (mi >> 1)), b0, b1, b2, b3);
          mma_bf16(o[n], pa, b0, b1);
          mma_bf16(o[n + 1], pa, b2, b3);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_bar[s]);  // this warp is done with stage s
    }
    q0 += ntiles;

    // quad-reduce the row sums
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);

    if (KG > 1) {
      // key groups 1..KG-1 hand (m, l, O) to key group 0 one after another
      // through the merge area ([row group][68 values][32 lanes]:
      // consecutive lanes, no conflicts); key group 0 merges them in order
      float* x = xs + (size_t)rg * 68 * 32 + lane;
      bool aborted = false;
      for (int k = 1; k < KG; ++k) {
        if (kg == k) {
#pragma unroll
          for (int n = 0; n < 16; ++n)
#pragma unroll
            for (int e = 0; e < 4; ++e) x[(n * 4 + e) * 32] = o[n][e];
          x[64 * 32] = m0;
          x[65 * 32] = m1;
          x[66 * 32] = l0;
          x[67 * 32] = l1;
        }
        // one decision for every consumer warp (the producer may set the
        // abort flag at any time; the barrier's AND is the same for all)
        if (!named_bar_and(1, NC * 32, !*(volatile int*)&s_abort)) {
          aborted = true;
          break;
        }
        if (kg == 0) {
          const float mk0 = x[64 * 32], mk1 = x[65 * 32];
          const float mn0 = fmaxf(m0, mk0), mn1 = fmaxf(m1, mk1);
          const float a0 = mn0 == -INFINITY ? 1.f : exp2f(m0 - mn0);
          const float a1 = mn1 == -INFINITY ? 1.f : exp2f(m1 - mn1);
          const float b0 = mn0 == -INFINITY ? 0.f : exp2f(mk0 - mn0);
          const float b1 = mn1 == -INFINITY ? 0.f : exp2f(mk1 - mn1);
#pragma unroll
          for (int n = 0; n < 16; ++n) {
            o[n][0] = o[n][0] * a0 + x[(n * 4 + 0) * 32] * b0;
            o[n][1] = o[n][1] * a0 + x[(n * 4 + 1) * 32] * b0;
            o[n][2] = o[n][2] * a1 + x[(n * 4 + 2) * 32] * b1;
            o[n][3] = o[n][3] * a1 + x[(n * 4 + 3) * 32] * b1;
          }
          l0 = l0 * a0 + x[66 * 32] * b0;
          l1 = l1 * a1 + x[67 * 32] * b1;
          m0 = mn0;
          m1 = mn1;
        }
        // the merge area is free again for the next key group / item
        named_bar_sync(1, NC * 32);
      }
      if (aborted) break;
      if (kg > 0) continue;
    } else if (*(volatile int*)&s_abort) {
      break;  // one warp per row group, no barrier among them: each decides alone
    }

    if (a.nsplit == 1) {
      // single split: normalise in place (same expression as the combine pass)
      const float inv0 = l0 > 0.f ? 1.0f / l0 : 0.f, inv1 = l1 > 0.f ? 1.0f / l1 : 0.f;
      if (v0) {
        bf16* dst = a.out + (((int64_t)b * a.T + t0) * a.Hq + kvh * a.G + r0 % a.G) * D;
#pragma unroll
        for (int n = 0; n < 16; ++n)
          *reinterpret_cast<uint32_t*>(dst + n * 8 + 2 * tig) = pack2(o[n][0] * inv0, o[n][1] * inv0);
      }
      if (v1) {
        bf16* dst = a.out + (((int64_t)b * a.T + t1) * a.Hq + kvh * a.G + r1 % a.G) * D;
#pragma unroll
        for (int n = 0; n < 16; ++n)
          *reinterpret_cast<uint32_t*>(dst + n * 8 + 2 * tig) = pack2(o[n][2] * inv1, o[n][3] * inv1);
      }
      continue;
    }
    float* wo = a.ws_o + unit * a.Rpad * D;
    float2* wml = a.ws_ml + unit * a.Rpad;
    if (v0) {
#pragma unroll
      for (int n = 0; n < 16; ++n)
        *reinterpret_cast<float2*>(wo + (int64_t)r0 * D + n * 8 + 2 * tig) = make_float2(o[n][0], o[n][1]);
      if (tig == 0) wml[r0] = make_float2(m0, l0);
    }
    if (v1) {
#pragma unroll
      for (int n = 0; n < 16; ++n)
        *reinterpret_cast<float2*>(wo + (int64_t)r1 * D + n * 8 + 2 * tig) = make_float2(o[n][2], o[n][3]);
      if (tig == 0) wml[r1] = make_float2(m1, l1);
    }
  }
}

// Merge the splits of one (b, kvh, row): splits with m = -inf hold nothing.
// Up to CMB_REG splits are loaded in one batch (every load in flight at
// once); the arithmetic - max over splits, then the weighted sum in split
// order - is the same for any split count.
constexpr int CMB_REG = 32;

__global__ void __launch_bounds__(128) attn_combine_kernel(AttnArgs a) {
  const int r = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int d = threadIdx.x;
  pdl_trigger();
  pdl_wait();
  const int t = r / a.G;
  const int start = a.starts[b];
  const int used = min(a.nsplit, (start + a.T + a.split_keys - 1) / a.split_keys);
  const int64_t base = ((int64_t)b * a.Hkv + kvh) * a.nsplit;
  float acc = 0.f, lsum = 0.f;
  if (used <= CMB_REG) {
    float2 ml[CMB_REG];
    float ov[CMB_REG];
#pragma unroll
    for (int s = 0; s < CMB_REG; ++s)
      if (s < used) {
        ml[s] = a.ws_ml[(base + s) * a.Rpad + r];
        ov[s] = a.ws_o[((base + s) * a.Rpad + r) * D + d];
      }
    float mmax = -INFINITY;
#pragma unroll
    for (int s = 0; s < CMB_REG; ++s)
      if (s < used) mmax = fmaxf(mmax, ml[s].x);
    if (mmax != -INFINITY) {
#pragma unroll
      for (int s = 0; s < CMB_REG; ++s)
        if (s < used && ml[s].x != -INFINITY) {
          const float w = exp2f(ml[s].x - mmax);
          lsum += w * ml[s].y;
          acc += w * ov[s];
        }
    }
  } else {
    float mmax = -INFINITY;
    for (int s = 0; s < used; ++s) mmax = fmaxf(mmax, a.ws_ml[(base + s) * a.Rpad + r].x);
    if (mmax != -INFINITY) {
      for (int s = 0; s < used; ++s) {
        const float2 ml = a.ws_ml[(base + s) * a.Rpad + r];
        if (ml.x == -INFINITY) continue;
        const float w = exp2f(ml.x - mmax);
        lsum += w * ml.y;
        acc += w * a.ws_o[((base + s) * a.Rpad + r) * D + d];
      }
    }
  }
  const float inv = lsum > 0.f ? 1.0f / lsum : 0.f;
  a.out[(((int64_t)b * a.T + t) * a.Hq + kvh * a.G + r % a.G) * D + d] = f2bf(acc * inv);
}

// key groups of a split: a function of split_keys alone (so a row's
// accumulation order never depends on the call's shape), each a divisor of
// ATT_STAGES.  Every key group has at least two ring stages, so a group
// computes one tile while its next one lands (with one stage per group each
// tile cost its compute plus the load's latency).  Splits of 768 keys or
// more spread over three warps, so a short context (one split) takes a few
// tiles per warp instead of a chain of them; shorter splits use two, which
// leaves room for three row groups, so a few query rows over a long context
// (decode, K+1 = 5) share each K/V tile within one CTA.
int attn_key_groups(int split_keys) {
  const int tiles = split_keys / TILE;
  return tiles >= 12 ? 3 : (tiles >= 2 ? 2 : 1);
}
static_assert(ATT_STAGES % 2 == 0 && ATT_STAGES % 3 == 0, "every key-group count must divide the ring depth");

// Row groups sharing the merge area: the ring's six 32 KB stages leave room
// for three row groups' slots within the 227 KB a CTA may use.
constexpr int ATT_MERGE_RG = 3;

// row groups per CTA: the most (up to ATT_MAX_WARPS / KG, and with key
// groups to merge up to ATT_MERGE_RG) that still give every SM a work item,
// else one (a short batch then spreads its rows over more CTAs; the K/V tiles
// they share come from L2).  Row blocks never change a row's arithmetic.
int attn_row_groups(int KG, int Rpad, long long per_rb_items, int num_sms) {
  const int groups = Rpad / 16;
  int cap = ATT_MAX_WARPS / KG;
  if (KG > 1 && cap > ATT_MERGE_RG) cap = ATT_MERGE_RG;
  int RG = cap < groups ? cap : groups;
  while (RG > 1 && per_rb_items * ((groups + RG - 1) / RG) < num_sms) RG /= 2;
  return RG;
}

// ring + merge area (one slot of 68 values per lane for each row group; the
// key groups take turns in it) + alignment
size_t attn_smem_bytes(int RG, int KG) {
  return 1024 + (size_t)ATT_STAGES * TILE_BYTES + (size_t)(KG > 1 ? RG : 0) * 68 * 32 * sizeof(float);
}

// the largest of any plan: ATT_MERGE_RG row groups' merge slots
size_t attn_smem_bytes_max() { return attn_smem_bytes(ATT_MERGE_RG, 2); }
static_assert(1024 + ATT_STAGES * TILE_BYTES + ATT_MERGE_RG * 68 * 32 * 4 + 512 <= 232448,
              "ring and merge area within a CTA's shared memory");

// ---------------------------------------------------------------------------
// tcgen05 variant: the same work units, split partials and combine pass, with
// both products on the 5th-generation tensor cores and the softmax run one
// thread per query row.
//
// * 192 threads.  Warp 0 (one lane) issues TMA loads of K and V tiles of 128
//   keys (two 64-dim boxes each, 128-byte swizzle) into a 2-deep ring;
//   warp 1 allocates TMEM and one lane issues the MMAs; warps 2-5 are the
//   128 query rows of the block (thread = row = TMEM lane).
// * S = Q K^T: M = 128 rows, N = 128 keys, K = 128 dims.  Q (staged by the
//   row threads) and K are both K-major in shared memory; S lands in one of
//   two TMEM buffers, so S of tile i+1 is computed while the rows run the
//   softmax of tile i.
// * Softmax: each thread reads its row of S from TMEM twice (row max, then
//   exp2 and row sum) and writes P (bf16) into shared memory in the
//   128-byte-swizzled K-major layout the next MMA reads.
// * O_i = P V: M = 128 rows, K = 128 keys, as two MMAs of N = 64 dims, each
//   reading one 64-dim box of the V tile MN-major (dims contiguous) straight
//   from TMA's layout.  Each thread folds its row of O_i into registers,
//   o = o * alpha + O_i: an online softmax over the tiles of the key split,
//   so one CTA can cover a long split without a combine pass.  P and O are
//   double-buffered and O_i is folded after the softmax of tile i+1, so the
//   P V product of one tile overlaps the softmax of the next.
// Masking, the log2-domain softmax and the partial layout are those of
// verify_attn_kernel, so the combine pass is shared.
// ---------------------------------------------------------------------------
constexpr int ATC_THREADS = 192;
constexpr int ATC_TILE = 128;                  // keys per tile
constexpr int ATC_BOX = ATC_TILE * 128;        // 128 rows x one 128-byte swizzle row: 16 KB
constexpr int ATC_REGION = 2 * ATC_BOX;        // 128 rows x 128 dims (or keys) in bf16: 32 KB
constexpr int ATC_STAGES = 2;
constexpr int ATC_TMEM_COLS = 512;             // S buffers at columns 0 and 128, O buffers at 256 and 384
constexpr int ATC_O_COL = 256;
// cluster mode: row partials [128][ATC_PO_LD] fp32 (rows padded by 16 bytes
// against bank conflicts) then (m, l) per row, in the idle K/V ring
constexpr int ATC_PO_LD = 132;
constexpr int ATC_PML_OFF = 128 * ATC_PO_LD * 4;
constexpr int ATC_MAX_CLUSTER = 8;              // portable cluster size
static_assert(ATC_PML_OFF + 128 * 8 <= ATC_STAGES * 2 * ATC_REGION, "cluster partials fit in the K/V ring");

struct AtcSmem {
  uint64_t k_full[ATC_STAGES];
  uint64_t v_full[ATC_STAGES];
  uint64_t kv_empty[ATC_STAGES];
  uint64_t s_full[2];
  uint64_t s_free[2];
  uint64_t p_full[2];
  uint64_t o_full[2];
  uint64_t o_free[2];
  uint64_t q_full;
  uint64_t drain_bar;  // abort path: completion of the MMAs issued so far
  uint32_t tmem_base;
  int abort;
};

// 32 consecutive TMEM columns of this thread's lane, one wait for the load
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ float2 ld_cluster_f2(uint32_t addr) {
  float2 v;
  asm volatile("ld.shared::cluster.v2.f32 {%0,%1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr) : "memory");
  return v;
}

__device__ __forceinline__ float4 ld_cluster_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// byte offset of 16-byte chunk c (of 16) of row `row` in a 128 x 128 bf16
// region stored as two 64-column boxes with the TMA 128-byte swizzle
__device__ __forceinline__ uint32_t atc_off(int row, int c) {
  return (c >> 3) * ATC_BOX + row * 128 + (((c & 7) ^ (row & 7)) << 4);
}

// Shared-memory descriptor of an MN-major operand of one 64-element swizzle
// atom along N (one 128-byte-swizzled row per K index, groups of 8 rows 1024
// bytes apart along K).  With a single atom along N the two strides of the
// descriptor have one meaning between them, the K-group stride, so both hold
// 1024.
__device__ __forceinline__ uint64_t sdesc_sw128_mn64(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)(1024 >> 4) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

__global__ void __launch_bounds__(ATC_THREADS, 1)
    verify_attn_tc_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                          AttnArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ AtcSmem sh;
  uint8_t* q_s = smem;                    // Q rows of the block, kept for every tile
  uint8_t* p_s = smem + ATC_REGION;       // P of tile i in buffer i & 1
  uint8_t* kv_s = smem + 3 * ATC_REGION;  // stage s: K at s * 2 * REGION, V after it
  // cluster mode: the nsplit splits of one row block are consecutive CTAs
  const int rb = a.cl ? blockIdx.x / a.nsplit : blockIdx.x % a.nrb;
  const int split = a.cl ? blockIdx.x % a.nsplit : blockIdx.x / a.nrb;
  const int kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ATC_STAGES; ++s) {
      mbar_init(&sh.k_full[s], 1);
      mbar_init(&sh.v_full[s], 1);
      mbar_init(&sh.kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sh.s_full[i], 1);
      mbar_init(&sh.s_free[i], 128);
    }
    mbar_init(&sh.q_full, 128);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sh.p_full[i], 128);
      mbar_init(&sh.o_full[i], 1);
      mbar_init(&sh.o_free[i], 128);
    }
    mbar_init(&sh.drain_bar, 1);
    sh.abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sh.tmem_base)),
                 "r"(ATC_TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  pdl_trigger();
  pdl_wait();
  const int start = a.starts[b];
  const int kv_len = start + a.T;
  // causal rows see no key past start + t: the block's last token bounds the
  // tiles it needs (a tile past it would only add exact zeros)
  int vis_end = kv_len;
  if (a.tree_mask == nullptr) vis_end = min(kv_len, start + (min(a.R, (rb + 1) * 128) - 1) / a.G + 1);
  const int key_begin = split * a.split_keys;
  const int key_end = min(key_begin + a.split_keys, vis_end);
  const int ntiles = key_end > key_begin ? (key_end - key_begin + ATC_TILE - 1) / ATC_TILE : 0;
  int issued = 0;  // producer lane: K/V tiles requested; MMA lane: 1 once an MMA was issued

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0 && ntiles > 0) {
      prefetch_tmap(&kmap);
      prefetch_tmap(&vmap);
      const int row0 = (int)(((int64_t)b * a.Hkv + kvh) * a.S) + key_begin;
      for (int i = 0; i < ntiles; ++i) {
        const int s = i % ATC_STAGES;
        if (i >= ATC_STAGES && !mbar_wait(&sh.kv_empty[s], ((i / ATC_STAGES) - 1) & 1)) {
          atomicExch(a.status, TSDS_E_TIMEOUT);
          sh.abort = 1;
          break;
        }
        if (*(volatile int*)&sh.abort) break;
        uint8_t* ks = kv_s + s * 2 * ATC_REGION;
        const int row = row0 + i * ATC_TILE;
        mbar_arrive_expect_tx(&sh.k_full[s], ATC_REGION);
        tma_load_2d(ks, &kmap, &sh.k_full[s], 0, row);
        tma_load_2d(ks + ATC_BOX, &kmap, &sh.k_full[s], 64, row);
        mbar_arrive_expect_tx(&sh.v_full[s], ATC_REGION);
        tma_load_2d(ks + ATC_REGION, &vmap, &sh.v_full[s], 0, row);
        tma_load_2d(ks + ATC_REGION + ATC_BOX, &vmap, &sh.v_full[s], 64, row);
        issued = i + 1;
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0 && ntiles > 0) {
      // bf16 x bf16 -> fp32, M = 128: S with N = 128 keys; O in two MMAs of
      // N = 64 dims (one V box each), B (V) read MN-major
      const uint32_t idesc_s = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(128 >> 3) << 17) |
                               ((uint32_t)(128 >> 4) << 24);
      const uint32_t idesc_o = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | ((uint32_t)(64 >> 3) << 17) |
                               ((uint32_t)(128 >> 4) << 24);
      const uint32_t qa = smem_u32(q_s), pa = smem_u32(p_s);
      auto issue_s = [&](int i) -> bool {
        const int s = i % ATC_STAGES, sb = i & 1;
        if (!mbar_wait(&sh.k_full[s], (i / ATC_STAGES) & 1)) return false;
        if (i >= 2 && !mbar_wait(&sh.s_free[sb], ((i - 2) >> 1) & 1)) return false;
        if (*(volatile int*)&sh.abort) return false;
        tc::tc_fence_after();
        const uint32_t kb = smem_u32(kv_s + s * 2 * ATC_REGION);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * ATC_BOX + (kk & 3) * 32;
          tc::umma_bf16(tmem + sb * 128, tc::sdesc_sw128(qa + off), tc::sdesc_sw128(kb + off), idesc_s,
                        kk > 0 ? 1u : 0u);
        }
        tc::umma_commit(&sh.s_full[sb]);
        issued = 1;
        return true;
      };
      bool ok = mbar_wait(&sh.q_full, 0) && issue_s(0);
      for (int i = 0; ok && i < ntiles; ++i) {
        if (i + 1 < ntiles && !issue_s(i + 1)) {
          ok = false;
          break;
        }
        const int s = i % ATC_STAGES, pb = i & 1;
        if (!mbar_wait(&sh.p_full[pb], (i >> 1) & 1) || !mbar_wait(&sh.v_full[s], (i / ATC_STAGES) & 1) ||
            (i >= 2 && !mbar_wait(&sh.o_free[pb], ((i - 2) >> 1) & 1)) || *(volatile int*)&sh.abort) {
          ok = false;
          break;
        }
        tc::tc_fence_after();
        const uint32_t vb = smem_u32(kv_s + s * 2 * ATC_REGION + ATC_REGION);
        const uint32_t pbuf = pa + pb * ATC_REGION;
#pragma unroll
        for (int h = 0; h < 2; ++h)  // dims 64h..64h+63: O columns 64h.., V box h
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)  // 16 keys per step: two 8-key groups of 1024 bytes
            tc::umma_bf16(tmem + ATC_O_COL + pb * 128 + h * 64,
                          tc::sdesc_sw128(pbuf + (kk >> 2) * ATC_BOX + (kk & 3) * 32),
                          sdesc_sw128_mn64(vb + h * ATC_BOX + kk * 2048), idesc_o, kk > 0 ? 1u : 0u);
        tc::umma_commit(&sh.kv_empty[s]);
        tc::umma_commit(&sh.o_full[pb]);
      }
      if (!ok) {
        atomicExch(a.status, TSDS_E_TIMEOUT);
        sh.abort = 1;
      }
    }
  } else {
    // ---------------- query rows (warps 2-5) ----------------
    const int eq = warp & 3;
    const int r = eq * 32 + lane;  // row of the block == TMEM lane
    const int row = rb * 128 + r;
    const bool valid = row < a.R;
    const int t = valid ? row / a.G : 0, gh = valid ? row % a.G : 0;
    {
      const bf16* qrow = a.q + (((int64_t)b * a.T + t) * a.Hq + kvh * a.G + gh) * D;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const uint4 v = valid ? *reinterpret_cast<const uint4*>(qrow + c * 8) : make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4*>(q_s + atc_off(r, c)) = v;
      }
    }
    fence_proxy_async();  // the MMA (async proxy) reads what these threads wrote
    mbar_arrive(&sh.q_full);
    // Visible keys of this row: every key below `lo`, and key mask_base + i
    // for each bit i of `mbits` - the causal rule (keys up to start + t) or
    // the tree rule (shared context below mask_base, then bit i of the row's
    // mask for key mask_base + i, nothing from mask_base + 32 on), both cut
    // at kv_len.
    int lo = 0, mask_base = 0;
    uint32_t mbits = 0u;
    if (valid) {
      if (a.tree_mask != nullptr) {
        mask_base = a.mask_origin >= 0 ? a.mask_origin : start;
        lo = min(mask_base, kv_len);
        const int span = kv_len - mask_base;  // keys from mask_base below kv_len
        mbits = span <= 0 ? 0u : (a.tree_mask[b * a.T + t] & (span >= 32 ? 0xffffffffu : ((1u << span) - 1u)));
      } else {
        lo = min(kv_len, start + t + 1);
      }
    }
    auto visible = [lo, mask_base, mbits](int kabs) {
      const uint32_t rel = (uint32_t)(kabs - mask_base);
      return kabs < lo || (rel < 32u && ((mbits >> (rel & 31u)) & 1u));
    };
    const uint32_t lane_off = (uint32_t)(eq * 32) << 16;
    float o[128];
#pragma unroll
    for (int i = 0; i < 128; ++i) o[i] = 0.f;
    float m = -INFINITY, l = 0.f;
    bool alive = true;
    // O_j = P_j V_j into o: o = o * alpha_j + O_j.  Runs after the softmax of
    // tile j + 1 (or after the last tile), so the P V product of one tile
    // overlaps the softmax of the next; the warp takes one decision.
    auto fold = [&](int j, float alpha) -> bool {
      const int ob = j & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&sh.o_full[ob], (j >> 1) & 1) ? 1 : 0)) {
        if (lane == 0) atomicExch(a.status, TSDS_E_TIMEOUT);
        sh.abort = 1;
        return false;
      }
      tc::tc_fence_after();
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float v[32];
        tmem_ld32(tmem + lane_off + ATC_O_COL + ob * 128 + c * 32, v);
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) o[c * 32 + jj] = o[c * 32 + jj] * alpha + v[jj];
      }
      tc::tc_fence_before();
      mbar_arrive(&sh.o_free[ob]);
      return true;
    };
    float al_prev = 1.f;
    for (int i = 0; i < ntiles; ++i) {
      const int sb = i & 1;
      // the warp takes one decision (tcgen05.ld is warp-collective)
      if (!__all_sync(0xffffffffu, mbar_wait(&sh.s_full[sb], (i >> 1) & 1) ? 1 : 0)) {
        if (lane == 0) atomicExch(a.status, TSDS_E_TIMEOUT);
        sh.abort = 1;
        alive = false;
        break;
      }
      tc::tc_fence_after();
      const int key0 = key_begin + i * ATC_TILE;
      const uint32_t sa = tmem + lane_off + sb * 128;
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float v[32];
        tmem_ld32(sa + c * 32, v);
#pragma unroll
        for (int j = 0; j < 32; ++j) mx = fmaxf(mx, visible(key0 + c * 32 + j) ? v[j] * a.scale_log2 : -INFINITY);
      }
      // rows with nothing visible so far keep m = -inf and p = 0
      const float mn = fmaxf(m, mx);
      const float al = mn == -INFINITY ? 1.f : exp2f(m - mn);
      const float sub = mn == -INFINITY ? 0.f : mn;
      m = mn;
      float ps = 0.f;
      uint8_t* pbuf = p_s + (i & 1) * ATC_REGION;  // free: O_{i-2}, its last reader, was folded
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        float v[16];
        tc::tmem_ld16(sa + c * 16, v);
        uint32_t pk[8];
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
          const float s0 = visible(key0 + c * 16 + j) ? v[j] * a.scale_log2 : -INFINITY;
          const float s1 = visible(key0 + c * 16 + j + 1) ? v[j + 1] * a.scale_log2 : -INFINITY;
          const float p0 = exp2f(s0 - sub), p1 = exp2f(s1 - sub);
          ps += p0 + p1;
          pk[j >> 1] = pack_bf2(p0, p1);
        }
        *reinterpret_cast<uint4*>(pbuf + atc_off(r, 2 * c)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        *reinterpret_cast<uint4*>(pbuf + atc_off(r, 2 * c + 1)) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
      }
      l = l * al + ps;
      tc::tc_fence_before();
      mbar_arrive(&sh.s_free[sb]);  // S buffer sb may be overwritten
      fence_proxy_async();
      mbar_arrive(&sh.p_full[i & 1]);
      if (i >= 1 && !fold(i - 1, al_prev)) {
        alive = false;
        break;
      }
      al_prev = al;
    }
    if (alive && ntiles > 0 && !fold(ntiles - 1, al_prev)) alive = false;
    if (a.cl) {
      // this row's partial into shared memory (the K/V ring is idle now)
      // for the cluster's combine below
      float* po = reinterpret_cast<float*>(kv_s) + r * ATC_PO_LD;
#pragma unroll
      for (int c = 0; c < 32; ++c)
        *reinterpret_cast<float4*>(po + 4 * c) = alive ? make_float4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3])
                                                       : make_float4(0.f, 0.f, 0.f, 0.f);
      reinterpret_cast<float2*>(kv_s + ATC_PML_OFF)[r] = alive ? make_float2(m, l) : make_float2(-INFINITY, 0.f);
    } else if (alive && valid) {
      if (a.nsplit == 1) {
        // single split: normalise in place (same expression as the combine pass)
        const float inv = l > 0.f ? 1.0f / l : 0.f;
        bf16* dst = a.out + (((int64_t)b * a.T + t) * a.Hq + kvh * a.G + gh) * D;
#pragma unroll
        for (int c = 0; c < 16; ++c)
          *reinterpret_cast<uint4*>(dst + c * 8) =
              make_uint4(pack_bf2(o[c * 8] * inv, o[c * 8 + 1] * inv), pack_bf2(o[c * 8 + 2] * inv, o[c * 8 + 3] * inv),
                         pack_bf2(o[c * 8 + 4] * inv, o[c * 8 + 5] * inv),
                         pack_bf2(o[c * 8 + 6] * inv, o[c * 8 + 7] * inv));
      } else {
        const int64_t unit = ((int64_t)b * a.Hkv + kvh) * a.nsplit + split;
        float4* wo = reinterpret_cast<float4*>(a.ws_o + (unit * a.Rpad + row) * D);
#pragma unroll
        for (int c = 0; c < 32; ++c) wo[c] = make_float4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
        a.ws_ml[unit * a.Rpad + row] = make_float2(m, l);
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (sh.abort) {  // uniform: read after the barrier
    // a CTA that gave up still lets its copies and MMAs in flight finish
    // (bounded) before TMEM is freed and it exits
    if (warp == 0 && lane == 0 && issued > 0) {
      drain_tma_ring(sh.k_full, ATC_STAGES, issued);
      drain_tma_ring(sh.v_full, ATC_STAGES, issued);
    }
    if (warp == 1 && lane == 0 && issued > 0) tc::drain_mma<1>(&sh.drain_bar);
    __syncthreads();
  }
  if (a.cl) {
    // Combine of the cluster's nsplit partials (the arithmetic and split
    // order of attn_combine_kernel): CTA `split` finishes rows
    // [split*128/n, (split+1)*128/n) of the block, a warp per row, a lane per
    // 4 dims, reading every CTA's partials through distributed shared memory.
    tc::cluster_sync_all();  // every CTA's partials are written
    const int n = a.nsplit;
    const uint32_t po0 = smem_u32(kv_s), pml0 = smem_u32(kv_s + ATC_PML_OFF);
    for (int rr = split * 128 / n + warp; rr < (split + 1) * 128 / n; rr += ATC_THREADS / 32) {
      const int row = rb * 128 + rr;
      if (row >= a.R) break;  // uniform over the warp
      float2 ml[ATC_MAX_CLUSTER];
      float mmax = -INFINITY;
#pragma unroll
      for (int q = 0; q < ATC_MAX_CLUSTER; ++q)
        if (q < n) {
          ml[q] = ld_cluster_f2(tc::mapa_shared(pml0 + rr * 8, q));
          mmax = fmaxf(mmax, ml[q].x);
        }
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      float lsum = 0.f;
      if (mmax != -INFINITY) {
#pragma unroll
        for (int q = 0; q < ATC_MAX_CLUSTER; ++q)
          if (q < n && ml[q].x != -INFINITY) {
            const float w = exp2f(ml[q].x - mmax);
            lsum += w * ml[q].y;
            const float4 v = ld_cluster_f4(tc::mapa_shared(po0 + (rr * ATC_PO_LD + 4 * lane) * 4, q));
            acc.x += w * v.x;
            acc.y += w * v.y;
            acc.z += w * v.z;
            acc.w += w * v.w;
          }
      }
      const float inv = lsum > 0.f ? 1.0f / lsum : 0.f;
      const int t = row / a.G, gh = row % a.G;
      bf16* dst = a.out + (((int64_t)b * a.T + t) * a.Hq + kvh * a.G + gh) * D + 4 * lane;
      *reinterpret_cast<uint2*>(dst) = make_uint2(pack_bf2(acc.x * inv, acc.y * inv), pack_bf2(acc.z * inv, acc.w * inv));
    }
    tc::cluster_sync_all();  // no CTA leaves while another still reads its shared memory
  }
  if (warp == 1) {
    tc::tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ATC_TMEM_COLS));
  }
}

// alignment + Q + two P buffers + the K/V ring
constexpr size_t atc_smem_bytes() { return 1024 + 3 * (size_t)ATC_REGION + (size_t)ATC_STAGES * 2 * ATC_REGION; }

// Process-wide switch for the tcgen05 variant (off by default; 2: with the
// clustered combine where the split count allows).
std::atomic<int> g_attn_tc{0};

// Whether clusters of n tcgen05-attention CTAs (a whole SM's shared memory
// each) can be resident; cached per n.
bool atc_clusters_fit(int n) {
  static std::atomic<int> known[ATC_MAX_CLUSTER + 1];  // 0 unknown, 1 yes, 2 no
  if (known[n].load(std::memory_order_acquire) == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(n);
    cfg.blockDim = dim3(ATC_THREADS);
    cfg.dynamicSmemBytes = atc_smem_bytes();
    cudaLaunchAttribute ca[1];
    ca[0].id = cudaLaunchAttributeClusterDimension;
    ca[0].val.clusterDim.x = n;
    ca[0].val.clusterDim.y = 1;
    ca[0].val.clusterDim.z = 1;
    cfg.attrs = ca;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, verify_attn_tc_kernel, &cfg) != cudaSuccess) {
      cudaGetLastError();
      clusters = 0;
    }
    known[n].store(clusters > 0 ? 1 : 2, std::memory_order_release);
  }
  return known[n].load(std::memory_order_acquire) == 1;
}

}  // namespace

// The default kernel's launch shape for a call (num_sms 0: the current
// device's): out = {RG, KG, row blocks, key splits, ring stages, threads}.
extern "C" int tsds_attention_plan(int B, int T, int Hq, int Hkv, int max_kv, int split_keys, int num_sms,
                                   int32_t* out) {
  TSDS_RETURN_IF(!out || B <= 0 || T <= 0 || Hq <= 0 || Hkv <= 0 || (Hq % Hkv) != 0, TSDS_E_INVALID);
  TSDS_RETURN_IF(max_kv <= 0 || split_keys <= 0 || (split_keys % TILE) != 0 || num_sms < 0, TSDS_E_INVALID);
  const long long R = (long long)T * (Hq / Hkv);
  TSDS_RETURN_IF(R > 1024, TSDS_E_UNSUPPORTED);
  const int Rpad = (int)((R + 15) / 16 * 16);
  const int KG = attn_key_groups(split_keys);
  const int nsplit = (max_kv + split_keys - 1) / split_keys;
  const int RG = attn_row_groups(KG, Rpad, (long long)B * Hkv * nsplit, num_sms > 0 ? num_sms : tsds_tc_num_sms());
  out[0] = RG;
  out[1] = KG;
  out[2] = (Rpad + RG * 16 - 1) / (RG * 16);
  out[3] = nsplit;
  out[4] = ATT_STAGES;
  out[5] = 32 * (1 + RG * KG);
  return TSDS_OK;
}

extern "C" void tsds_set_attention_tc(int mode) { g_attn_tc = mode < 0 ? 0 : (mode > 2 ? 2 : mode); }
extern "C" int tsds_get_attention_tc(void) { return g_attn_tc; }

extern "C" size_t tsds_attention_workspace_bytes(int B, int T, int Hq, int Hkv, int Dd, int max_kv, int split_keys) {
  if (B <= 0 || T <= 0 || Hkv <= 0 || Hq % Hkv || Dd != D || split_keys <= 0) return 0;
  const int R = T * (Hq / Hkv);
  const int Rpad = (R + 15) / 16 * 16;
  const int nsplit = (max_kv + split_keys - 1) / split_keys;
  if (nsplit <= 1) return 0;
  return (size_t)B * Hkv * nsplit * Rpad * (D * sizeof(float) + sizeof(float2));
}

extern "C" int tsds_verify_attention(const void* q, const void* k_cache, const void* v_cache, void* out,
                                     const int32_t* starts, const uint32_t* tree_mask, int mask_origin, int B, int T,
                                     int Hq, int Hkv, int Dd, int S, int max_kv, int split_keys, float scale,
                                     void* workspace, size_t workspace_bytes, int32_t* status, tsds_stream_t stream) {
  TSDS_RETURN_IF(Dd != D, TSDS_E_UNSUPPORTED);
  TSDS_RETURN_IF(B <= 0 || T <= 0 || Hq <= 0 || Hkv <= 0 || (Hq % Hkv) != 0 || S <= 0, TSDS_E_INVALID);
  TSDS_RETURN_IF(tree_mask != nullptr && mask_origin < 0 && T > 32, TSDS_E_INVALID);
  TSDS_RETURN_IF(max_kv <= 0 || max_kv > S || split_keys <= 0 || (split_keys % TILE) != 0, TSDS_E_INVALID);
  TSDS_RETURN_IF(!q || !k_cache || !v_cache || !out || !starts || !status, TSDS_E_INVALID);
  TSDS_RETURN_IF(!tsds_aligned16(q) || !tsds_aligned16(k_cache) || !tsds_aligned16(v_cache) || !tsds_aligned16(out),
                 TSDS_E_ALIGN);
  const int G = Hq / Hkv;
  const long long R64 = (long long)T * G;
  // the tcgen05 variant takes any number of 128-row blocks (a prompt's rows
  // in one call); the default kernel up to 1024 rows per kv head
  const bool tc = g_attn_tc && split_keys % ATC_TILE == 0;
  TSDS_RETURN_IF(R64 > (tc ? 65536 : 1024), TSDS_E_UNSUPPORTED);
  TSDS_RETURN_IF((uint64_t)B * Hkv * S > (uint64_t)INT32_MAX, TSDS_E_UNSUPPORTED);  // cache rows are int
  const int R = (int)R64;
  const int Rpad = (R + 15) / 16 * 16;
  // default kernel: row blocks of RG 16-row groups, KG key groups per split
  const int KG = attn_key_groups(split_keys);
  const int nsplit = (max_kv + split_keys - 1) / split_keys;
  const int RG = attn_row_groups(KG, Rpad, (long long)B * Hkv * nsplit, tsds_tc_num_sms());
  const int nrb = tc ? (Rpad + 127) / 128 : (Rpad + RG * 16 - 1) / (RG * 16);
  const size_t need = tsds_attention_workspace_bytes(B, T, Hq, Hkv, Dd, max_kv, split_keys);
  TSDS_RETURN_IF(need > workspace_bytes || (need > 0 && workspace == nullptr), TSDS_E_WORKSPACE);

  CUtensorMap kmap, vmap;
  const uint64_t rows = (uint64_t)B * Hkv * S;
  int st = tsds_make_tmap_2d_bf16(&kmap, k_cache, D, rows, D * 2, 64, TILE, 1);
  if (st != TSDS_OK) return st;
  st = tsds_make_tmap_2d_bf16(&vmap, v_cache, D, rows, D * 2, 64, TILE, 1);
  if (st != TSDS_OK) return st;

  AttnArgs a;
  a.q = (const bf16*)q;
  a.out = (bf16*)out;
  a.starts = starts;
  a.tree_mask = tree_mask;
  a.ws_o = (float*)workspace;
  a.ws_ml = nsplit > 1 ? reinterpret_cast<float2*>((char*)workspace + (size_t)B * Hkv * nsplit * Rpad * D * sizeof(float))
                       : nullptr;
  a.status = status;
  a.B = B;
  a.T = T;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.S = S;
  a.G = G;
  a.R = R;
  a.Rpad = Rpad;
  a.nsplit = nsplit;
  a.split_keys = split_keys;
  a.nrb = nrb;
  a.mask_origin = mask_origin;
  a.scale_log2 = scale * LOG2E;
  a.cl = 0;
  a.RG = RG;
  a.KG = KG;
  a.paged = 0;
  a.k_pool = a.v_pool = nullptr;
  a.table = nullptr;
  a.req_rows = nullptr;
  a.table_ld = a.pool_rows = 0;

  if (tc) {
    // 128-key boxes for the tcgen05 variant
    st = tsds_make_tmap_2d_bf16(&kmap, k_cache, D, rows, D * 2, 64, ATC_TILE, 1);
    if (st != TSDS_OK) return st;
    st = tsds_make_tmap_2d_bf16(&vmap, v_cache, D, rows, D * 2, 64, ATC_TILE, 1);
    if (st != TSDS_OK) return st;
    static tsds_device_flags tc_attr;
    st = tsds_smem_limit_once(verify_attn_tc_kernel, (int)atc_smem_bytes(), tc_attr);
    if (st != TSDS_OK) return st;
    if (g_attn_tc == 2 && nsplit >= 2 && nsplit <= ATC_MAX_CLUSTER && atc_clusters_fit(nsplit)) {
      // the splits of a row block as one cluster, combined in shared memory
      a.cl = 1;
      tsds_launch_cluster(verify_attn_tc_kernel, dim3(nrb * nsplit, Hkv, B), dim3(ATC_THREADS), atc_smem_bytes(),
                          stream, nsplit, kmap, vmap, a);
      return tsds_launch_status();
    }
    tsds_launch(verify_attn_tc_kernel, dim3(nsplit * nrb, Hkv, B), dim3(ATC_THREADS), atc_smem_bytes(), stream,
                kmap, vmap, a);
    st = tsds_launch_status();
    if (st != TSDS_OK || nsplit == 1) return st;
    tsds_launch(attn_combine_kernel, dim3(R, Hkv, B), dim3(128), 0, stream, a);
    return tsds_launch_status();
  }

  const size_t smem = attn_smem_bytes(RG, KG);
  static tsds_device_flags attr_set;
  st = tsds_smem_limit_once(verify_attn_kernel<ATT_STAGES>, (int)attn_smem_bytes_max(), attr_set);
  if (st != TSDS_OK) return st;
  // persistent: one CTA per SM (fewer when there are fewer work items)
  const long long items = (long long)B * Hkv * nrb * nsplit;
  TSDS_RETURN_IF(items > INT32_MAX, TSDS_E_UNSUPPORTED);
  const int grid = (int)(items < tsds_tc_num_sms() ? items : tsds_tc_num_sms());
  tsds_launch(verify_attn_kernel<ATT_STAGES>, dim3(grid), dim3(32 * (1 + RG * KG)), smem, stream, kmap, vmap, a);
  st = tsds_launch_status();
  if (st != TSDS_OK || nsplit == 1) return st;
  tsds_launch(attn_combine_kernel, dim3(R, Hkv, B), dim3(128), 0, stream, a);
  return tsds_launch_status();
}

// ---------------------------------------------------------------------------
// Verify attention over paged token pools (SGLang's token_to_kv_pool layout:
// per layer K and V pools [pool_rows][Hkv][D], a request-to-token table
// giving the pool row of every position of a sequence).  The default
// kernel's work items, masks, key groups and split partials, with the K/V
// tiles staged from the pools: by TMA when pages hold a multiple of 64
// tokens (each aligned run of 64 keys is 64 consecutive pool rows), else
// gathered row by row by the producer warp.  The arithmetic is the
// contiguous path's, so a sequence gives bit-identical outputs whichever
// layout holds its keys.
// ---------------------------------------------------------------------------
extern "C" int tsds_verify_attention_paged(const void* q, const void* k_pool, const void* v_pool, void* out,
                                           const int32_t* starts, const uint32_t* tree_mask, int mask_origin,
                                           const int32_t* token_table, int64_t table_ld, const int64_t* req_rows,
                                           int64_t pool_rows, int page_size, int B, int T, int Hq, int Hkv, int Dd,
                                           int max_kv, int split_keys, float scale, void* workspace,
                                           size_t workspace_bytes, int32_t* status, tsds_stream_t stream) {
  TSDS_RETURN_IF(Dd != D, TSDS_E_UNSUPPORTED);
  TSDS_RETURN_IF(B <= 0 || T <= 0 || Hq <= 0 || Hkv <= 0 || (Hq % Hkv) != 0, TSDS_E_INVALID);
  TSDS_RETURN_IF(tree_mask != nullptr && mask_origin < 0 && T > 32, TSDS_E_INVALID);
  TSDS_RETURN_IF(max_kv <= 0 || max_kv > table_ld || split_keys <= 0 || (split_keys % TILE) != 0, TSDS_E_INVALID);
  TSDS_RETURN_IF(pool_rows <= 0 || page_size <= 0 || pool_rows > (int64_t)INT32_MAX, TSDS_E_INVALID);
  TSDS_RETURN_IF(!q || !k_pool || !v_pool || !out || !starts || !status || !token_table, TSDS_E_INVALID);
  TSDS_RETURN_IF(!tsds_aligned16(q) || !tsds_aligned16(k_pool) || !tsds_aligned16(v_pool) || !tsds_aligned16(out),
                 TSDS_E_ALIGN);
  const int G = Hq / Hkv;
  const long long R64 = (long long)T * G;
  TSDS_RETURN_IF(R64 > 1024, TSDS_E_UNSUPPORTED);
  const int R = (int)R64;
  const int Rpad = (R + 15) / 16 * 16;
  const int KG = attn_key_groups(split_keys);
  const int nsplit = (max_kv + split_keys - 1) / split_keys;
  const int RG = attn_row_groups(KG, Rpad, (long long)B * Hkv * nsplit, tsds_tc_num_sms());
  const int nrb = (Rpad + RG * 16 - 1) / (RG * 16);
  const size_t need = tsds_attention_workspace_bytes(B, T, Hq, Hkv, Dd, max_kv, split_keys);
  TSDS_RETURN_IF(need > workspace_bytes || (need > 0 && workspace == nullptr), TSDS_E_WORKSPACE);

  AttnArgs a;
  a.q = (const bf16*)q;
  a.out = (bf16*)out;
  a.starts = starts;
  a.tree_mask = tree_mask;
  a.ws_o = (float*)workspace;
  a.ws_ml = nsplit > 1 ? reinterpret_cast<float2*>((char*)workspace + (size_t)B * Hkv * nsplit * Rpad * D * sizeof(float))
                       : nullptr;
  a.status = status;
  a.B = B;
  a.T = T;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.S = table_ld < (int64_t)INT32_MAX ? (int)table_ld : INT32_MAX;
  a.G = G;
  a.R = R;
  a.Rpad = Rpad;
  a.nsplit = nsplit;
  a.split_keys = split_keys;
  a.nrb = nrb;
  a.mask_origin = mask_origin;
  a.scale_log2 = scale * LOG2E;
  a.cl = 0;
  a.RG = RG;
  a.KG = KG;
  a.paged = page_size % TILE == 0 ? 1 : 2;
  a.k_pool = (const bf16*)k_pool;
  a.v_pool = (const bf16*)v_pool;
  a.table = token_table;
  a.req_rows = req_rows;
  a.table_ld = table_ld;
  a.pool_rows = pool_rows;

  CUtensorMap kmap, vmap;
  memset(&kmap, 0, sizeof(kmap));
  memset(&vmap, 0, sizeof(vmap));
  if (a.paged == 1) {
    // the pools as [pool_rows][Hkv * D]: a box is 64 pool rows x one 64-column half of a kv head
    int st = tsds_make_tmap_2d_bf16(&kmap, k_pool, (uint64_t)Hkv * D, (uint64_t)pool_rows, (uint64_t)Hkv * D * 2, 64,
                                    TILE, 1);
    if (st != TSDS_OK) return st;
    st = tsds_make_tmap_2d_bf16(&vmap, v_pool, (uint64_t)Hkv * D, (uint64_t)pool_rows, (uint64_t)Hkv * D * 2, 64,
                                TILE, 1);
    if (st != TSDS_OK) return st;
  }
  static tsds_device_flags attr_set;
  int st = tsds_smem_limit_once(verify_attn_kernel<ATT_STAGES>, (int)attn_smem_bytes_max(), attr_set);
  if (st != TSDS_OK) return st;
  const long long items = (long long)B * Hkv * nrb * nsplit;
  TSDS_RETURN_IF(items > INT32_MAX, TSDS_E_UNSUPPORTED);
  const int grid = (int)(items < tsds_tc_num_sms() ? items : tsds_tc_num_sms());
  tsds_launch(verify_attn_kernel<ATT_STAGES>, dim3(grid), dim3(32 * (1 + RG * KG)), attn_smem_bytes(RG, KG), stream,
              kmap, vmap, a);
  st = tsds_launch_status();
  if (st != TSDS_OK || nsplit == 1) return st;
  tsds_launch(attn_combine_kernel, dim3(R, Hkv, B), dim3(128), 0, stream, a);
  return tsds_launch_status();
}

// ---------------------------------------------------------------------------
// Verify attention for callers that cannot allocate device memory.
//
// Some callers of this library run where they may not call cudaMalloc: a
// plugin inside a serving framework that reserved the device memory for
// itself up front (SGLang sizes its KV pool to a fixed fraction of the GPU
// and leaves nothing for extensions), or code that must not allocate while
// a stream is being captured into a graph.  This entry point needs no
// workspace from them: its split-KV partials live in the file-scope array
// below, a fixed 8 MiB (plus a 256-byte header holding the status word)
// that every GPU which loads the library keeps until the process exits.
//
// * Host code never passes the array's name to a kernel (on the host that
//   name is only a stand-in, not a device address).  The first call on a
//   device, with that device current, looks up the device address with
//   cudaGetSymbolAddress and caches it with the current context; a call in
//   another context (after cudaDeviceReset) looks it up again.  Make the
//   first call on a device (and the first after a reset) before any stream
//   capture.
// * All calls share the array and it keeps the last call's contents: the
//   status word is cleared at each call (the partials are fully rewritten
//   before they are read), and calls that overlap on the GPU race with
//   each other.  Order them on one stream.
// * A request whose partials exceed the 8 MiB returns TSDS_E_SCRATCH_LIMIT.
// ---------------------------------------------------------------------------
namespace {
constexpr size_t kNoAllocHeader = 256;
constexpr size_t kNoAllocScratch = size_t(8) << 20;
constexpr int kNoAllocMaxDevices = 64;
}  // namespace

static __device__ __align__(256) unsigned char g_attn_noalloc_scratch[kNoAllocHeader + kNoAllocScratch];

// The array's device address per device, with the context it was looked up
// in: after cudaDeviceReset (or any re-creation of the primary context) the
// module is loaded again, possibly elsewhere, so a changed current context
// means a fresh lookup.
struct NoAllocAddr {
  void* ctx;
  void* ptr;
};
static NoAllocAddr g_attn_noalloc_addr[kNoAllocMaxDevices];
static std::mutex g_attn_noalloc_lock;

typedef int (*CtxGetCurrentFn)(void**);

static void* current_context() {
  static std::atomic<CtxGetCurrentFn> fn{nullptr};
  CtxGetCurrentFn f = fn.load(std::memory_order_acquire);
  if (f == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || p == nullptr) {
      cudaGetLastError();
      return nullptr;
    }
    f = reinterpret_cast<CtxGetCurrentFn>(p);
    fn.store(f, std::memory_order_release);
  }
  void* ctx = nullptr;
  return f(&ctx) == 0 ? ctx : nullptr;
}

static int attn_noalloc_base(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return TSDS_E_DEVICE;
  }
  if (dev < 0 || dev >= kNoAllocMaxDevices) return TSDS_E_DEVICE;
  std::lock_guard<std::mutex> hold(g_attn_noalloc_lock);
  NoAllocAddr& c = g_attn_noalloc_addr[dev];
  // no context current yet (this thread's first CUDA work): the lookup below
  // makes the device's primary context current
  void* ctx = current_context();
  if (c.ptr == nullptr || ctx == nullptr || c.ctx != ctx) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return TSDS_E_DEVICE;
    }
    ctx = current_context();
    if (ctx == nullptr) return TSDS_E_DEVICE;
    c.ptr = p;
    c.ctx = ctx;
  }
  *out = c.ptr;
  return TSDS_OK;
}

extern "C" size_t tsds_verify_attention_noalloc_limit(void) { return kNoAllocScratch; }

extern "C" int tsds_verify_attention_noalloc(const void* q, const void* k_cache, const void* v_cache, void* out,
                                             const int32_t* starts, const uint32_t* tree_mask, int mask_origin, int B,
                                             int T, int Hq, int Hkv, int Dd, int S, int max_kv, int split_keys,
                                             float scale, tsds_stream_t stream) {
  const size_t need = tsds_attention_workspace_bytes(B, T, Hq, Hkv, Dd, max_kv, split_keys);
  if (need > kNoAllocScratch) return TSDS_E_SCRATCH_LIMIT;
  void* base = nullptr;
  const int st = attn_noalloc_base(&base);
  if (st != TSDS_OK) return st;
  int32_t* status = static_cast<int32_t*>(base);
  if (cudaMemsetAsync(status, 0, sizeof(int32_t), stream) != cudaSuccess) {
    cudaGetLastError();
    return TSDS_E_LAUNCH;
  }
  return tsds_verify_attention(q, k_cache, v_cache, out, starts, tree_mask, mask_origin, B, T, Hq, Hkv, Dd, S, max_kv,
                               split_keys, scale, static_cast<char*>(base) + kNoAllocHeader, kNoAllocScratch, status,
                               stream);
}

extern "C" int tsds_verify_attention_noalloc_status(int32_t* host_status) {
  void* base = nullptr;
  const int st = attn_noalloc_base(&base);
  if (st != TSDS_OK) return st;
  if (host_status == nullptr) return TSDS_E_INVALID;
  if (cudaMemcpy(host_status, base, sizeof(int32_t), cudaMemcpyDeviceToHost) != cudaSuccess) {
    cudaGetLastError();
    return TSDS_E_DEVICE;
  }
  return TSDS_OK;
}
