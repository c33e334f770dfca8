// Multi-stage residual VQ on CTA pairs: the two CTAs of a cluster hold the
// same rows and split every stage's codebook between them.
//
// Why a pair.  The tensor-core MMA is 128 rows tall (one TMEM lane per row).
// A batch of 8192 frames spread over 148 SMs gives 56 rows per SM, so a CTA
// that owns its rows for the whole codebook leaves more than half of every
// MMA on empty lanes, and each stage's MMAs wait for the stage's serial
// resolve.  Here a pair holds up to 128 rows (8192 frames -> 74 pairs of
// 111 rows on 148 SMs) and each CTA computes the dots of half the codes
// (codebook tiles [0, ceil(T/2)) on rank 0, the rest on rank 1), so a stage
// costs each SM half the tensor time at full lane use.
//
// The selection is unchanged: every CTA screens its own codes with the TF32
// window of rvq_tc.cu (relative to the maximum over its own codes, which
// still contains every minimiser among them) and resolves its candidates
// with the exact pinned arithmetic, or scans its codes exactly when a row's
// preconditions fail or its records overflow.  The result per row is one
// 64-bit key, (orderable exact distance << 32) | code, with a NaN distance
// keyed below every number (first NaN wins) and -0 mapped to +0; the smaller
// of the two CTAs' keys is the first minimum over all codes, i.e. exactly
// the code of rvq_tc_kernel and of the FFMA kernel.
//
// Exchange.  Each owner thread stores its row's key straight into the
// peer's shared memory (st.async, counted in bytes on the peer's mbarrier
// of that stage parity) and waits for the peer's key on its own mbarrier.
// The expected byte count of stage s + 2 is posted when stage s ends, before
// any key of stage s + 1 leaves, so the peer cannot run ahead of it.  At
// teardown each CTA tells its peer how many stages of keys it sent, and
// each waits (bounded) until those keys have landed before the pair exits,
// so no store is in flight into a CTA that has left, timeouts included.
//
// Roles (320 threads): warps 0-7 epilogue (row = TMEM lane (warp % 4) * 32 +
// lane, column half warp / 4 of every 256-code tile; the half-0 thread owns
// the row: residual in registers, resolve, update, the next A operand),
// warp 8 producer (bulk copies of this CTA's codebook tile images), warp 9
// TMEM allocator and MMA issuer.  Rank 0 writes the codes and the
// reconstruction, rank 1 the residual.  Every wait is bounded.
#include "rvq_tc.cuh"

namespace moss {
namespace rvqtc {

struct __align__(1024) PairSmem {
  float btile[kSlots][kTileBytes / 4];  // tile images (each 1024-aligned)
  float a[kRows * kDim];                // 2r, K-major SW128 image
  float a_extra[kRows * 8];             // [1, 0 x 7] per row, no-swizzle K block
  // Per screening slot (column half x row):
  float rec_max[kRec][2 * kRows];
  uint32_t rec_mask[kRec][2 * kRows];
  unsigned char rec_chunk[kRec][2 * kRows];
  float amax_h[2 * kRows];
  int nrec_h[2 * kRows];
  float window[kRows];
  int pre_slow[kRows];
  int row_bad[kRows];
  unsigned long long best[kRows];      // this CTA's key per row
  unsigned long long xbest[2][kRows];  // the peer's keys, by stage parity
  int queue[kEpiThreads / 32][kQueue];  // (row << 16) | code
  float norms[kRows];
  int slow_list[kRows];
  int slow_count;
  int peer_sent;  // stages of keys the peer sent (written by the peer at teardown)
  uint32_t tmem_base;
  alignas(8) unsigned long long b_full[kSlots];
  alignas(8) unsigned long long b_empty[kSlots];
  alignas(8) unsigned long long t_full[2];
  alignas(8) unsigned long long t_empty[2];
  alignas(8) unsigned long long a_full;
  alignas(8) unsigned long long x_full[2];  // the peer's keys of stage parity 0 / 1 landed
};
static_assert(sizeof(PairSmem) + 1024 <= 232448, "shared memory above the sm_100 per-block limit");

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t peer_addr(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
// 8 bytes into the peer's shared memory, counted on the peer's mbarrier.
__device__ __forceinline__ void st_async_u64(uint32_t addr, unsigned long long v, uint32_t bar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.b64 [%0], %1, [%2];" ::"r"(addr),
      "l"(v), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void st_cluster_u32(uint32_t addr, int v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

// The selection key of an exact distance: smaller is better, the code breaks
// ties (first minimum); a NaN distance keys below every number (first NaN).
__device__ __forceinline__ unsigned long long dist_key(float dist, int j) {
  if (dist != dist) return static_cast<unsigned long long>(static_cast<uint32_t>(j));
  return (static_cast<unsigned long long>(order_key(__fadd_rn(dist, 0.0f))) << 32) |
         static_cast<uint32_t>(j);
}

// Exact NaN-aware selection of one row over codes [lo, hi) by one warp, as a
// key (the pinned arithmetic of exact_scan).
__device__ unsigned long long exact_scan_key(const float* tw, float norm,
                                             const float* __restrict__ book,
                                             const float* __restrict__ cnorm, int lo, int hi,
                                             int lane) {
  unsigned long long best = ~0ull;
  for (int j = lo + lane; j < hi; j += 32) {
    const float* c = book + static_cast<int64_t>(j) * kDim;
    float dot = 0.0f;
    for (int d = 0; d < kDim; ++d) dot = __fmaf_rn(tw[d], c[d], dot);
    const unsigned long long key = dist_key(__fadd_rn(__fsub_rn(norm, dot), cnorm[j]), j);
    best = key < best ? key : best;
  }
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) {
    const unsigned long long o = __shfl_xor_sync(0xffffffffu, best, m);
    best = o < best ? o : best;
  }
  return best;
}

__global__ void __launch_bounds__(kThreads, 1) rvq_pair_kernel(Args a) {
  extern __shared__ unsigned char smem_raw[];
  PairSmem& sm = *reinterpret_cast<PairSmem*>(
      smem_raw +
      ((1024u - (static_cast<uint32_t>(__cvta_generic_to_shared(smem_raw)) & 1023u)) & 1023u));
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_rank();
  const uint32_t peer = rank ^ 1u;
  const int ntiles = a.kpad / kTileCodes;  // >= 2
  const int half_tiles = (ntiles + 1) / 2;
  const int t_lo = rank == 0 ? 0 : half_tiles;
  const int nloc = rank == 0 ? half_tiles : ntiles - half_tiles;
  const int code_lo = t_lo * kTileCodes;
  const int code_hi = min(a.k, (t_lo + nloc) * kTileCodes);
  const int total_tiles = a.stages * nloc;
  const int rpc = a.rows_per_cta;  // rows of the pair, <= 128
  const int64_t row0 = static_cast<int64_t>(blockIdx.x >> 1) * rpc;
  const uint32_t xbytes = static_cast<uint32_t>(rpc) * 8u;

  if (tid == 0) {
    for (int i = 0; i < kSlots; ++i) {
      mbar_init(&sm.b_full[i], 1);
      mbar_init(&sm.b_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.t_full[i], 1);
      mbar_init(&sm.t_empty[i], kEpiThreads);
      mbar_init(&sm.x_full[i], 1);
    }
    mbar_init(&sm.a_full, kRows);  // every owner thread writes its lane
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    sm.slow_count = 0;
    sm.peer_sent = 0;
    // the peer's keys of stages 0 and 1
    mbar_arrive_expect_tx(&sm.x_full[0], xbytes);
    if (a.stages > 1) mbar_arrive_expect_tx(&sm.x_full[1], xbytes);
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&sm.tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  // both CTAs' barriers are initialised before any key crosses
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  int sent = 0;  // stages whose keys this CTA sent (tracked by thread 0)

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      for (int q = 0; q < total_tiles; ++q) {
        const int slot = q % kSlots;
        const int s = q / nloc, t = q - s * nloc;
        if (!mbar_wait(&sm.b_empty[slot], ((q / kSlots) & 1) ^ 1)) break;
        mbar_arrive_expect_tx(&sm.b_full[slot], kTileBytes);
        bulk_g2s(&sm.btile[slot][0],
                 a.image + (static_cast<int64_t>(s) * ntiles + t_lo + t) * (kTileBytes / 4),
                 kTileBytes, &sm.b_full[slot]);
      }
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t a_base = smem_u32(sm.a);
      const uint64_t a_extra = plain_desc(smem_u32(sm.a_extra));
      int q = 0;
      bool ok = true;
      for (int s = 0; s < a.stages && ok; ++s) {
        if (!mbar_wait(&sm.a_full, s & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int t = 0; t < nloc; ++t, ++q) {
          const int slot = q % kSlots;
          const int abuf = q & 1;
          if (!mbar_wait(&sm.b_full[slot], (q / kSlots) & 1) ||
              !mbar_wait(&sm.t_empty[abuf], ((q >> 1) & 1) ^ 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t b_base = smem_u32(&sm.btile[slot][0]);
          const uint32_t d_tmem = tmem + static_cast<uint32_t>(abuf * 256);
#pragma unroll
          for (int kk = 0; kk < kDim / 8; ++kk) {
            const uint32_t koff = static_cast<uint32_t>(kk >> 2);
            const uint64_t ad =
                sw128_desc(a_base + koff * (kRows * 128u) + static_cast<uint32_t>(kk & 3) * 32u);
            const uint64_t bd = sw128_desc(b_base + koff * (kTileCodes * 128u) +
                                           static_cast<uint32_t>(kk & 3) * 32u);
            mma_tf32(d_tmem, ad, bd, kk > 0 ? 1u : 0u);
          }
          // 9th K step: 1 x (-cnorm_j)
          mma_tf32(d_tmem, a_extra, plain_desc(b_base + kMainBytes), 1u);
          mma_commit(&sm.t_full[abuf]);
          mma_commit(&sm.b_empty[slot]);
        }
      }
      // Let the final commit arrivals land before the CTA can retire.
      for (int last = (q > kSlots ? q - kSlots : 0); ok && last < q; ++last) {
        ok = mbar_wait(&sm.b_empty[last % kSlots], (last / kSlots) & 1);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int lr = quarter * 32 + lane;  // local row = TMEM lane
    const int part = warp >> 2;          // column half of every tile
    const int slot = part * kRows + lr;
    const bool owner = part == 0;
    const int64_t grow = row0 + lr;
    const bool valid = lr < rpc && grow < a.rows;
    float r[kDim];
    if (owner && valid) {
      const float4* src = reinterpret_cast<const float4*>(a.x + grow * kDim);
#pragma unroll
      for (int i = 0; i < kDim / 4; ++i) {
        const float4 v = src[i];
        r[4 * i] = v.x; r[4 * i + 1] = v.y; r[4 * i + 2] = v.z; r[4 * i + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int d = 0; d < kDim; ++d) r[d] = 0.0f;
    }
    unsigned char* a_bytes = reinterpret_cast<unsigned char*>(sm.a);
    if (owner) {
      unsigned char* e = reinterpret_cast<unsigned char*>(sm.a_extra);
#pragma unroll
      for (int k = 0; k < 8; ++k)
        *reinterpret_cast<float*>(e + plain_offset(lr, k)) = k == 0 ? 1.0f : 0.0f;
    }
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    auto write_a = [&]() {
      const uint32_t a_base = smem_u32(sm.a);
#pragma unroll
      for (int c = 0; c < kDim / 4; ++c) {
        const float x0 = __fmul_rn(2.0f, r[4 * c]), x1 = __fmul_rn(2.0f, r[4 * c + 1]);
        const float x2 = __fmul_rn(2.0f, r[4 * c + 2]), x3 = __fmul_rn(2.0f, r[4 * c + 3]);
        st_shared_v4(a_base + sw128_offset(lr, 4 * c, kRows * 128u), x0, x1, x2, x3);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(&sm.a_full);
    };
    if (owner) write_a();
    const uint32_t x_remote0 = peer_addr(smem_u32(&sm.x_full[0]), peer);
    const uint32_t x_remote1 = peer_addr(smem_u32(&sm.x_full[1]), peer);

    int q = 0;
    bool aborted = false;
    float next_cn_max = a.stats[0], next_flag = a.stats[1];
    for (int s = 0; s < a.stages; ++s) {
      const float* book = a.books + static_cast<int64_t>(s) * a.k * kDim;
      const float* cnorm = a.code_norm + static_cast<int64_t>(s) * a.kpad;
      const float cn_max = next_cn_max;
      const bool book_ok = next_flag == 0.0f;
      if (s + 1 < a.stages) {
        next_cn_max = a.stats[(s + 1) * 4 + 0];
        next_flag = a.stats[(s + 1) * 4 + 1];
      }
      if (owner) {
        float norm = 0.0f;
#pragma unroll
        for (int d = 0; d < kDim; ++d) norm = __fmaf_rn(r[d], r[d], norm);
        sm.norms[lr] = norm;
        // screening window and preconditions (rvq_tc.cu)
        const float sc = __fmul_rn(2.0f, sqrtf(norm)) * sqrtf(cn_max);
        const bool slow = !(isfinite(norm) && book_ok && sc < 1.0e36f);
        const float margin = sc * 0.00390625f + cn_max * 0.001953125f +
                             (norm + cn_max) * 9.5367431640625e-07f + 1e-30f;
        sm.window[lr] = 2.0f * margin * 1.0001f;
        sm.pre_slow[lr] = slow || !valid ? 1 : 0;
        sm.row_bad[lr] = 0;
        sm.best[lr] = ~0ull;
      }
      epi_bar();  // the window is visible to both column halves
      const float window = sm.window[lr];
      float amax = -CUDART_INF_F;
      int nrec = 0;
      int timed_out = 0;
      for (int t = 0; t < nloc; ++t, ++q) {
        const int abuf = q & 1;
        if (!timed_out && !mbar_wait(&sm.t_full[abuf], (q >> 1) & 1)) timed_out = 1;
        tc_fence_after();
        const uint32_t tcol = tmem + lane_base + static_cast<uint32_t>(abuf * 256 + part * 128);
        const int cbase = (t_lo + t) * 8 + part * 4;  // this thread's first 32-code chunk
#pragma unroll 1
        for (int c = 0; c < 4; c += 2) {
          uint32_t va[32], vb[32];
          tmem_load32(tcol + static_cast<uint32_t>(c * 32), va);
          tmem_load32(tcol + static_cast<uint32_t>((c + 1) * 32), vb);
          tmem_wait_ld(va);
          tmem_wait_ld(vb);
          if (c == 2) {
            // the accumulator is in registers: the MMA of the tile after
            // next may overwrite it
            tc_fence_before();
            mbar_arrive(&sm.t_empty[abuf]);
          }
          const float ca = max32(va), cb = max32(vb);
          amax = fmaxf(amax, fmaxf(ca, cb));
          const float athr = amax - window;
          const uint32_t ma = valid ? mask32(va, athr) : 0u;
          const uint32_t mb = valid ? mask32(vb, athr) : 0u;
          if (ma) nrec = add_record(sm, slot, cbase + c, ma, ca, athr, nrec);
          if (mb) nrec = add_record(sm, slot, cbase + c + 1, mb, cb, athr, nrec);
        }
      }
      sm.amax_h[slot] = amax;
      sm.nrec_h[slot] = nrec;
      if (epi_bar_or(timed_out)) {  // both halves' records are complete
        aborted = true;
        break;
      }

      // ---- resolve this CTA's candidates exactly (rvq_tc.cu)
      bool fast = sm.pre_slow[lr] == 0 && sm.nrec_h[lr] <= kRec && sm.nrec_h[kRows + lr] <= kRec;
      const float gmax = fmaxf(sm.amax_h[lr], sm.amax_h[kRows + lr]);
      const float athr = gmax - window;
      int slow_flag = (owner && valid && !fast) ? 1 : 0;
      int cnt = 0;
      int c0 = 0, c1 = 0, c2 = 0, c3 = 0;
      if (fast) {
        float rmax[kRec];
        uint32_t rmask[kRec];
#pragma unroll
        for (int e = 0; e < kRec; ++e) {
          rmax[e] = e < nrec ? sm.rec_max[e][slot] : -CUDART_INF_F;
          rmask[e] = e < nrec ? sm.rec_mask[e][slot] : 0u;
        }
#pragma unroll
        for (int e = 0; e < kRec; ++e) {
          if (rmax[e] < athr || rmask[e] == 0u) continue;
          const int base = sm.rec_chunk[e][slot] * 32;
          for (uint32_t m = rmask[e]; m; m &= m - 1) {
            const int j = base + (__ffs(m) - 1);
            if (cnt < 4) {
              const int jc = j < a.k ? j : 0;
              prefetch_l1(book + static_cast<int64_t>(jc) * kDim);
              prefetch_l1(book + static_cast<int64_t>(jc) * kDim + 32);
              c3 = cnt == 3 ? j : c3;
              c2 = cnt == 2 ? j : c2;
              c1 = cnt == 1 ? j : c1;
              c0 = cnt == 0 ? j : c0;
            }
            ++cnt;
          }
        }
      }
      int incl = cnt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      const int total = __shfl_sync(0xffffffffu, incl, 31);
      int* queue = sm.queue[warp];
      if (incl > kQueue) {
        sm.row_bad[lr] = 1;  // does not fit: exact scan
        slow_flag = 1;
      } else if (cnt > 4) {  // rare: walk the records again
        int pos = incl - cnt;
        for (int e = 0; e < nrec; ++e) {
          if (sm.rec_max[e][slot] < athr) continue;
          const int base = sm.rec_chunk[e][slot] * 32;
          for (uint32_t m = sm.rec_mask[e][slot]; m; m &= m - 1)
            queue[pos++] = (lr << 16) | (base + (__ffs(m) - 1));
        }
      } else if (cnt > 0) {
        const int pos = incl - cnt;
        queue[pos] = (lr << 16) | c0;
        if (cnt > 1) queue[pos + 1] = (lr << 16) | c1;
        if (cnt > 2) queue[pos + 2] = (lr << 16) | c2;
        if (cnt > 3) queue[pos + 3] = (lr << 16) | c3;
      }
      const int nq =
          total <= kQueue ? total : __reduce_max_sync(0xffffffffu, incl <= kQueue ? incl : 0);
      __syncwarp();
      for (int i = lane; i < nq; i += 32) {
        const int ent = queue[i];
        const int rr = ent >> 16, j = ent & 0xffff;
        if (j >= a.k) continue;  // padding columns never reach the window
        const float4* cw = reinterpret_cast<const float4*>(book + static_cast<int64_t>(j) * kDim);
        float4 w[kDim / 4];
#pragma unroll
        for (int i4 = 0; i4 < kDim / 4; ++i4) w[i4] = cw[i4];
        const float nj = cnorm[j];
        float dot = 0.0f;
#pragma unroll
        for (int i4 = 0; i4 < kDim / 4; ++i4) {
          const float4 tw =
              *reinterpret_cast<const float4*>(a_bytes + sw128_offset(rr, 4 * i4, kRows * 128u));
          dot = __fmaf_rn(tw.x, w[i4].x, dot);
          dot = __fmaf_rn(tw.y, w[i4].y, dot);
          dot = __fmaf_rn(tw.z, w[i4].z, dot);
          dot = __fmaf_rn(tw.w, w[i4].w, dot);
        }
        // fast rows have finite distances (their preconditions held)
        atomicMin(&sm.best[rr], dist_key(__fadd_rn(__fsub_rn(sm.norms[rr], dot), nj), j));
      }
      if (epi_bar_or(slow_flag)) {
        if (owner && valid && !(fast && sm.row_bad[lr] == 0)) {
          const int at = atomicAdd(&sm.slow_count, 1);
          sm.slow_list[at] = lr;
        }
        epi_bar();
        const int nslow = sm.slow_count;
        // exact scan of this CTA's codes, one warp per row; 2r is read back
        // from the A image
        for (int i = warp; i < nslow; i += kEpiThreads / 32) {
          const int sr = sm.slow_list[i];
          float tw[kDim];
          for (int d = 0; d < kDim; ++d)
            tw[d] = *reinterpret_cast<const float*>(a_bytes + sw128_offset(sr, d, kRows * 128u));
          const unsigned long long key =
              exact_scan_key(tw, sm.norms[sr], book, cnorm, code_lo, code_hi, lane);
          if (lane == 0) sm.best[sr] = key;
        }
        epi_bar();
        if (warp == 0 && lane == 0) sm.slow_count = 0;
      }

      // ---- exchange the keys with the peer; the smaller one wins
      int xfail = 0;
      unsigned long long key = ~0ull;
      if (owner && lr < rpc) {
        key = sm.best[lr];
        st_async_u64(peer_addr(smem_u32(&sm.xbest[s & 1][lr]), peer), key, (s & 1) ? x_remote1 : x_remote0);
        if (mbar_wait(&sm.x_full[s & 1], (s >> 1) & 1)) {
          const unsigned long long other = sm.xbest[s & 1][lr];
          key = other < key ? other : key;
        } else {
          xfail = 1;
        }
      }
      sent = s + 1;
      if (epi_bar_or(xfail)) {
        aborted = true;
        break;
      }
      if (owner && valid) {
        int winner = static_cast<int>(key & 0xffffffffull);
        if (key == ~0ull || winner >= a.k) {
          // Unreachable: each CTA's screening maximum is one of its real
          // codes, so every unflagged row has a resolved candidate in both
          // halves.  Kept in bounds, reported.
          record_device_error(MOSS_ERR_UNSUPPORTED);
          winner = 0;
        }
        const float4* cw =
            reinterpret_cast<const float4*>(book + static_cast<int64_t>(winner) * kDim);
#pragma unroll
        for (int i = 0; i < kDim / 4; ++i) {
          const float4 v = cw[i];
          r[4 * i] = __fsub_rn(r[4 * i], v.x);
          r[4 * i + 1] = __fsub_rn(r[4 * i + 1], v.y);
          r[4 * i + 2] = __fsub_rn(r[4 * i + 2], v.z);
          r[4 * i + 3] = __fsub_rn(r[4 * i + 3], v.w);
        }
        if (rank == 0) a.codes[static_cast<int64_t>(s) * a.rows + grow] = winner;
      }
      if (owner && s + 1 < a.stages) write_a();
      // every reader of this stage's A image, records and peer keys is done
      epi_bar();
      // the peer's keys of stage s + 2 land in this parity's buffer; the
      // count is posted before any key of stage s + 1 leaves this CTA
      if (tid == 0 && s + 2 < a.stages) mbar_arrive_expect_tx(&sm.x_full[s & 1], xbytes);
    }
    if (owner && !aborted && valid) {
      if (rank == 0) {
        // recon = sum of the chosen codewords in stage order from +0
        float acc[kDim];
#pragma unroll
        for (int d = 0; d < kDim; ++d) acc[d] = 0.0f;
#pragma unroll 4
        for (int s = 0; s < a.stages; ++s) {
          const int c = a.codes[static_cast<int64_t>(s) * a.rows + grow];
          const float4* cw = reinterpret_cast<const float4*>(
              a.books + (static_cast<int64_t>(s) * a.k + c) * kDim);
#pragma unroll
          for (int i = 0; i < kDim / 4; ++i) {
            const float4 v = cw[i];
            acc[4 * i] = __fadd_rn(acc[4 * i], v.x);
            acc[4 * i + 1] = __fadd_rn(acc[4 * i + 1], v.y);
            acc[4 * i + 2] = __fadd_rn(acc[4 * i + 2], v.z);
            acc[4 * i + 3] = __fadd_rn(acc[4 * i + 3], v.w);
          }
        }
        float4* dst = reinterpret_cast<float4*>(a.recon + grow * kDim);
#pragma unroll
        for (int i = 0; i < kDim / 4; ++i)
          dst[i] = make_float4(acc[4 * i], acc[4 * i + 1], acc[4 * i + 2], acc[4 * i + 3]);
      } else if (a.residual_out) {
        float4* res = reinterpret_cast<float4*>(a.residual_out + grow * kDim);
#pragma unroll
        for (int i = 0; i < kDim / 4; ++i)
          res[i] = make_float4(r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]);
      }
    }
  }

  // ---- teardown: every key sent into a CTA has landed before the pair exits
  if (tid == 0) st_cluster_u32(peer_addr(smem_u32(&sm.peer_sent), peer), sent);
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();
  if (tid == 0) {
    const int ps = sm.peer_sent;
    for (int b = 0; b < 2; ++b) {
      // the last stage of this parity whose keys the peer sent
      const int last = ps - 1 - ((ps - 1 - b) & 1);
      if (last >= 0) mbar_wait(&sm.x_full[b], (last >> 1) & 1, 100000000ull);
    }
  }
  __syncthreads();
  cluster_sync_all();
  tc_fence_after();
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}

}  // namespace rvqtc

// Pairs of the pair kernel that fit on the current device at once (cached
// per device); 0 when clusters of two cannot be placed.
int rvq_pair_capacity(size_t smem) {
  static int cached[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 0;
  if (cached[dev] != 0) return cached[dev] < 0 ? 0 : cached[dev];
  int n = 0;
  if (cudaFuncSetAttribute(rvqtc::rvq_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) == cudaSuccess) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(2 * (sm_count() / 2)), 1, 1);
    cfg.blockDim = dim3(rvqtc::kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, rvqtc::rvq_pair_kernel, &cfg) != cudaSuccess) n = 0;
  }
  cudaGetLastError();  // a refused query leaves no sticky error behind
  cached[dev] = n > 0 ? n : -1;
  return n > 0 ? n : 0;
}

// Launches the pair kernel over `pairs` clusters of two CTAs.
int launch_rvq_pair(const rvqtc::Args& args, int64_t pairs, void* stream) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs), 1, 1);
  cfg.blockDim = dim3(rvqtc::kThreads, 1, 1);
  cfg.dynamicSmemBytes = sizeof(rvqtc::PairSmem) + 1024;
  cfg.stream = as_stream(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, rvqtc::rvq_pair_kernel, args);
  if (e != cudaSuccess)
    return fail(MOSS_ERR_CUDA, "moss_rvq_encode: pair launch failed: %s", cudaGetErrorString(e));
  return launch_status("moss_rvq_encode");
}

size_t rvq_pair_smem() { return sizeof(rvqtc::PairSmem) + 1024; }

}  // namespace moss
