// Multi-stage residual VQ with tensor-core screening (tcgen05, TF32) and an
// exact FP32 resolution.  Produces exactly the codes of the FFMA kernel in
// rvq.cu (same documented arithmetic).
//
// Why the indices stay exact.  For row r and code j the tensor cores compute
//   acc_j = TF32 sum_d 2r_d c_jd  -  TF32(cnorm_j)      (9th K step: 1 x -cnorm)
// and key_j = -acc_j approximates exact_j = dist_j - norm (real-number
// difference; dist_j in the pinned FP32 order of rvq.cu).  TF32 keeps 10
// fraction bits (relative error < 2^-10 per operand), so the products are
// within 2^-9 sum|2r_d c_jd| <= 2^-9 S C (S = |2r|, C = max_j |c_j|) and the
// folded norm within 2^-10 cnorm_max; the pinned FP32 dot and the two FP32
// roundings of dist add less than 2^-20 (norm + cnorm_max + S C).  Hence
//   |key_j - exact_j| <= M = 2^-8 S C + 2^-9 cnorm_max + 2^-20 (norm + cnorm_max)
// (twice the TF32 bound).  Every minimiser j* of dist has key_j* <= min key
// + 2M, so the candidates {j : acc_j >= max acc - 2M} contain all of them.
// One candidate is the answer; several are resolved with the exact pinned
// arithmetic (first minimum wins).  Rows whose preconditions fail
// (non-finite norm or codebook, S C >= 1e36, candidate records overflow) are
// resolved by an exact NaN-aware scan of all codes.
//
// SIMT shape of the screening: per 32-code chunk a thread (one row) takes the
// chunk maximum, updates its running maximum, and forms a 32-bit mask of the
// codes inside the window -- all branch-free.  Only a non-empty mask costs a
// (rare, short) record of {chunk, mask, chunk max} in shared memory; the
// records are filtered against the final window at the end of the stage.
//
// This kernel gives one CTA its rows for the whole codebook; rvq_pair.cu
// splits each codebook over a CTA pair and is used wherever it applies (at
// least two 256-code tiles, the rows within one wave of pairs).  Here a CTA
// owns `rows_per_cta` rows for all stages, 320 threads:
//   warps 0-7  epilogue (256 threads).  With at most 64 rows per CTA (while
//              the rows fit one CTA per SM: e.g. 8192 rows -> 147 CTAs of
//              56) every row is written into two TMEM lanes (lane i
//              and 64 + i), so four threads screen its 256 columns per tile
//              (two lane copies x two column halves); with 128 rows per CTA
//              each row has one lane and two threads.  The part-0 thread of
//              a row owns its norm, window and slow-path flag; the lanes of
//              each warp share the exact resolve of its candidate queue; the
//              residual itself is spread over all 256 threads in 16-byte
//              units (16 adjacent lanes per row), which update it and write
//              the next stage's A operand (2r, K-major 128B-swizzled);
//   warp 8     producer: cp.async.bulk of pre-built 256-code codebook tile
//              images (64 KB swizzled dims + 8 KB norm column) into 2 slots;
//   warp 9     TMEM allocator + MMA issuer: per tile 9 x tcgen05.mma
//              (M=128, N=256, K=8) into one of two 256-column accumulators.
// Every wait is bounded (~2 s) and records MOSS_ERR_TIMEOUT; all roles then
// meet at the final barrier where the TMEM is released.
#include "rvq_tc.cuh"

namespace moss {
namespace rvqtc {

struct __align__(1024) Smem {
  float btile[kSlots][kTileBytes / 4];  // tile images (each 1024-aligned)
  float a[kRows * kDim];                // 2r, K-major SW128 image
  float a_extra[kRows * 8];             // [1, 0 x 7] per row, no-swizzle K block
  // Per screening slot (column part x local row, at most 256 slots):
  float cmax[4][2 * kRows];  // chunk maxima of the current tile
  float rec_max[kRec][2 * kRows];
  uint32_t rec_mask[kRec][2 * kRows];
  unsigned char rec_chunk[kRec][2 * kRows];
  float amax_h[2 * kRows];  // running screening maximum
  int nrec_h[2 * kRows];
  float window[kRows];
  int pre_slow[kRows];  // row fails the screening preconditions this stage
  int row_bad[kRows];   // row's candidates did not fit the resolve queue
  unsigned long long best[kRows];  // (orderable distance << 32) | code
  int queue[kEpiThreads / 32][kQueue];  // (row << 16) | code
  float norms[kRows];
  int sel[kRows];
  int slow_list[kRows];
  int slow_count;
  uint32_t tmem_base;
  alignas(8) unsigned long long b_full[kSlots];
  alignas(8) unsigned long long b_empty[kSlots];
  alignas(8) unsigned long long t_full[2];
  alignas(8) unsigned long long t_empty[2];
  alignas(8) unsigned long long a_full;
};
// The dynamic allocation adds 1024 bytes of alignment slack.
static_assert(sizeof(Smem) + 1024 <= 232448, "shared memory above the sm_100 per-block limit");

// kCopies = 2: at most 64 rows per CTA, every row in two TMEM lanes; 1: up to
// 128 rows, one lane each.
template <int kCopies>
__global__ void __launch_bounds__(kThreads, 1) rvq_tc_kernel(Args a) {
  extern __shared__ unsigned char smem_raw[];
  // 1024-byte alignment for the swizzled operand images, by pointer
  // arithmetic on the shared array: the compiler then keeps the shared state
  // space for every access through `sm` (an integer round trip would turn
  // them into generic accesses).
  Smem& sm = *reinterpret_cast<Smem*>(
      smem_raw +
      ((1024u - (static_cast<uint32_t>(__cvta_generic_to_shared(smem_raw)) & 1023u)) & 1023u));
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int ntiles = a.kpad / kTileCodes;
  const int total_tiles = a.stages * ntiles;
  const int rpc = a.rows_per_cta;
  // rows_per_cta <= 64: every row sits in two TMEM lanes, copy c of local
  // row i in lane c * 64 + i (lanes i >= rpc of each copy hold no row)
  constexpr int copies = kCopies;
  const int span = kRows / copies;  // lanes per copy
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * rpc;

  if (tid == 0) {
    for (int i = 0; i < kSlots; ++i) {
      mbar_init(&sm.b_full[i], 1);
      mbar_init(&sm.b_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.t_full[i], 1);
      mbar_init(&sm.t_empty[i], kEpiThreads);
    }
    mbar_init(&sm.a_full, kEpiThreads);  // every epilogue thread writes its units
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    sm.slow_count = 0;
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
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      for (int q = 0; q < total_tiles; ++q) {
        const int slot = q % kSlots;
        if (!mbar_wait(&sm.b_empty[slot], ((q / kSlots) & 1) ^ 1)) break;
        mbar_arrive_expect_tx(&sm.b_full[slot], kTileBytes);
        bulk_g2s(&sm.btile[slot][0], a.image + static_cast<int64_t>(q) * (kTileBytes / 4),
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
        for (int t = 0; t < ntiles; ++t, ++q) {
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
    // The CTA's rpc rows sit in the 128 TMEM lanes `copies` times (lane L
    // holds local row L % span when that is below rpc).  Warp w reads the lanes of quarter w % 4, and
    // the 2 * copies warps that see a row split every tile's 256 columns
    // into equal parts.  The part-0 thread of a row owns it (residual in
    // registers): it writes the A operand, resolves and updates.
    const int quarter = warp & 3;
    const int qpr = 4 / copies;               // lane quarters per copy
    const int lr = (quarter % qpr) * 32 + lane;  // local row
    const int part = (quarter / qpr) * 2 + (warp >> 2);
    const int nparts = 2 * copies;
    const int cpp = 8 / nparts;               // 32-code chunks per part and tile
    const int slot = part * span + lr;
    const bool owner = part == 0;
    const int64_t grow = row0 + lr;
    const bool valid = lr < rpc && grow < a.rows;
    // The residual is spread over all epilogue threads in 16-byte units: unit
    // i of thread `tid` is dims [4 uchunk, 4 uchunk + 4) of local row
    // unit_row(i), so the 16 units of a row sit in 16 adjacent lanes and each
    // codeword read, A-image write and output store of a row is one
    // contiguous 256-byte span.
    constexpr int kUnits = kRows / kCopies * (kDim / 4) / kEpiThreads;
    const int uchunk = tid & 15;
    auto unit_row = [&](int i) { return (tid >> 4) + 16 * i; };
    auto unit_valid = [&](int i) { return unit_row(i) < rpc && row0 + unit_row(i) < a.rows; };
    float4 r4[kUnits];
#pragma unroll
    for (int i = 0; i < kUnits; ++i) {
      r4[i] = unit_valid(i)
                  ? reinterpret_cast<const float4*>(a.x + (row0 + unit_row(i)) * kDim)[uchunk]
                  : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    unsigned char* a_bytes = reinterpret_cast<unsigned char*>(sm.a);
    if (owner) {
      unsigned char* e = reinterpret_cast<unsigned char*>(sm.a_extra);
      for (int cp = 0; cp < copies; ++cp) {
#pragma unroll
        for (int k = 0; k < 8; ++k)
          *reinterpret_cast<float*>(e + plain_offset(lr + cp * span, k)) = k == 0 ? 1.0f : 0.0f;
      }
    }
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    // The A operand (2r, in every copy) of the next stage is written as soon
    // as the residual is known, so that its MMA starts before the bookkeeping
    // of the stage boundary.  Every epilogue thread writes its units (rows
    // past the CTA's rows hold zeros) and arrives.
    const uint32_t a_base = smem_u32(sm.a);
    auto write_a = [&]() {
#pragma unroll
      for (int i = 0; i < kUnits; ++i) {
        const float x0 = __fmul_rn(2.0f, r4[i].x), x1 = __fmul_rn(2.0f, r4[i].y);
        const float x2 = __fmul_rn(2.0f, r4[i].z), x3 = __fmul_rn(2.0f, r4[i].w);
        st_shared_v4(a_base + sw128_offset(unit_row(i), 4 * uchunk, kRows * 128u), x0, x1, x2, x3);
        if (kCopies == 2)
          st_shared_v4(a_base + sw128_offset(unit_row(i) + span, 4 * uchunk, kRows * 128u), x0, x1,
                       x2, x3);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(&sm.a_full);
    };
    write_a();
    epi_bar();  // the first A image is complete before the owners read it

    int q = 0;
    bool aborted = false;
    // The stage's codebook statistics are loaded one stage ahead.
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
      float norm = 0.0f;
      if (owner) {
        // r_d = (2 r_d) / 2 exactly from the A image; where 2 r_d overflowed,
        // r_d^2 overflows as well, so the sum is the same
#pragma unroll
        for (int c = 0; c < kDim / 4; ++c) {
          const float4 tw =
              *reinterpret_cast<const float4*>(a_bytes + sw128_offset(lr, 4 * c, kRows * 128u));
          const float r0 = __fmul_rn(0.5f, tw.x), r1 = __fmul_rn(0.5f, tw.y);
          const float r2 = __fmul_rn(0.5f, tw.z), r3 = __fmul_rn(0.5f, tw.w);
          norm = __fmaf_rn(r0, r0, norm);
          norm = __fmaf_rn(r1, r1, norm);
          norm = __fmaf_rn(r2, r2, norm);
          norm = __fmaf_rn(r3, r3, norm);
        }
        sm.norms[lr] = norm;
        sm.sel[lr] = -1;  // set by the exact scan for the rows that take it
        // screening window and preconditions
        const float sc = __fmul_rn(2.0f, sqrtf(norm)) * sqrtf(cn_max);
        const bool slow = !(isfinite(norm) && book_ok && sc < 1.0e36f);
        const float margin = sc * 0.00390625f + cn_max * 0.001953125f +
                             (norm + cn_max) * 9.5367431640625e-07f + 1e-30f;
        sm.window[lr] = 2.0f * margin * 1.0001f;
        sm.pre_slow[lr] = slow || !valid ? 1 : 0;
        sm.row_bad[lr] = 0;
        sm.best[lr] = ~0ull;
      }
      epi_bar();  // the window is visible to every part
      const float window = sm.window[lr];
      float amax = -CUDART_INF_F;
      int nrec = 0;
      // A timed-out wait is agreed on at the end of the stage (all threads
      // run the same tiles; after a timeout this thread stops waiting and
      // the stage's values are discarded).
      int timed_out = 0;
      for (int t = 0; t < ntiles; ++t, ++q) {
        const int abuf = q & 1;
        if (!timed_out && !mbar_wait_spin(&sm.t_full[abuf], (q >> 1) & 1)) timed_out = 1;
        tc_fence_after();
        const uint32_t tcol =
            tmem + lane_base + static_cast<uint32_t>(abuf * 256 + part * cpp * 32);
        uint32_t va[32], vb[32];
        if (cpp == 2) {
          // 64 rows per CTA: the part's two chunks are loaded once and kept
          // in registers for the mask.
          tmem_load32(tcol, va);
          tmem_load32(tcol + 32u, vb);
          tmem_wait_ld(va);
          tmem_wait_ld(vb);
          // The accumulator is in registers: hand it back to the MMA warp
          // now, so that the tile after next is computed while this one is
          // screened.
          tc_fence_before();
          mbar_arrive(&sm.t_empty[abuf]);
          const float ca = max32(va), cb = max32(vb);
          amax = fmaxf(amax, fmaxf(ca, cb));
          const float athr = amax - window;
          const uint32_t ma = valid ? mask32(va, athr) : 0u;
          const uint32_t mb = valid ? mask32(vb, athr) : 0u;
          const int chunk = t * 8 + part * cpp;
          if (ma) nrec = add_record(sm, slot, chunk, ma, ca, athr, nrec);
          if (mb) nrec = add_record(sm, slot, chunk + 1, mb, cb, athr, nrec);
        } else {
          // Pass 1: the chunk maxima of this part of the tile, then one
          // threshold; pass 2: window masks of the chunks that reach it.
          float tmax = -CUDART_INF_F;
#pragma unroll 1
          for (int c = 0; c < cpp; c += 2) {
            tmem_load32(tcol + static_cast<uint32_t>(c * 32), va);
            tmem_load32(tcol + static_cast<uint32_t>((c + 1) * 32), vb);
            tmem_wait_ld(va);
            tmem_wait_ld(vb);
            const float ca = max32(va), cb = max32(vb);
            sm.cmax[c][slot] = ca;
            sm.cmax[c + 1][slot] = cb;
            tmax = fmaxf(tmax, fmaxf(ca, cb));
          }
          amax = fmaxf(amax, tmax);
          const float athr = amax - window;
#pragma unroll 1
          for (int c = 0; c < cpp; c += 2) {
            tmem_load32(tcol + static_cast<uint32_t>(c * 32), va);
            tmem_load32(tcol + static_cast<uint32_t>((c + 1) * 32), vb);
            tmem_wait_ld(va);
            tmem_wait_ld(vb);
            const uint32_t ma = valid ? mask32(va, athr) : 0u;
            const uint32_t mb = valid ? mask32(vb, athr) : 0u;
            const int chunk = t * 8 + part * cpp + c;
            if (ma) nrec = add_record(sm, slot, chunk, ma, sm.cmax[c][slot], athr, nrec);
            if (mb) nrec = add_record(sm, slot, chunk + 1, mb, sm.cmax[c + 1][slot], athr, nrec);
          }
          tc_fence_before();
          mbar_arrive(&sm.t_empty[abuf]);
        }
      }
      sm.amax_h[slot] = amax;
      sm.nrec_h[slot] = nrec;
      if (epi_bar_or(timed_out)) {  // every part's records are complete
        aborted = true;
        break;
      }

      // ---- resolve the stage: every surviving candidate gets its exact
      // distance.  The lanes of a warp share the candidates of its 32 rows
      // (from the A image, 2r in shared memory); per row the smallest
      // (distance, code) key wins, i.e. the first minimum.
      bool fast = sm.pre_slow[lr] == 0;
      float gmax = -CUDART_INF_F;
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        if (p < nparts) {
          fast = fast && sm.nrec_h[p * span + lr] <= kRec;
          gmax = fmaxf(gmax, sm.amax_h[p * span + lr]);
        }
      }
      const float athr = gmax - window;
      // A row needs the exact scan when its preconditions failed or its
      // candidates overflow the queue; the flag rides on the next barrier.
      int slow_flag = (owner && valid && !fast) ? 1 : 0;
      // The records' fields are loaded together and filtered without
      // branches; each record keeps its mask if its chunk maximum is still
      // inside the final window.
      int cnt = 0;
      uint32_t keep[kRec];
      int base[kRec];
#pragma unroll
      for (int e = 0; e < kRec; ++e) {
        const bool live = fast && e < nrec;
        const float mx = live ? sm.rec_max[e][slot] : -CUDART_INF_F;
        const uint32_t mask = live ? sm.rec_mask[e][slot] : 0u;
        base[e] = live ? sm.rec_chunk[e][slot] * 32 : 0;
        keep[e] = mx >= athr ? mask : 0u;
        cnt += __popc(keep[e]);
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
      } else if (cnt > 0) {
        int pos = incl - cnt;
#pragma unroll
        for (int e = 0; e < kRec; ++e) {
          for (uint32_t m = keep[e]; m; m &= m - 1u)
            queue[pos++] = (lr << 16) | (base[e] + (__ffs(m) - 1));
        }
      }
      // entries [0, nq) are written: the rows whose candidates all fit
      const int nq = total <= kQueue ? total : __reduce_max_sync(0xffffffffu, incl <= kQueue ? incl : 0);
      __syncwarp();
      for (int i = lane; i < nq; i += 32) {
        const int ent = queue[i];
        const int rr = ent >> 16, j = ent & 0xffff;
        if (j >= a.k) continue;  // padding columns never reach the window
        const float4* cw = reinterpret_cast<const float4*>(book + static_cast<int64_t>(j) * kDim);
        float4 w[kDim / 4];
#pragma unroll
        for (int i4 = 0; i4 < kDim / 4; ++i4) w[i4] = cw[i4];
        // the code norm in the prepared order (sequential FMAs from +0), from
        // the codeword in registers instead of one more dependent load
        float nj = 0.0f;
        float dot = 0.0f;
#pragma unroll
        for (int i4 = 0; i4 < kDim / 4; ++i4) {
          const float4 tw =
              *reinterpret_cast<const float4*>(a_bytes + sw128_offset(rr, 4 * i4, kRows * 128u));
          dot = __fmaf_rn(tw.x, w[i4].x, dot);
          dot = __fmaf_rn(tw.y, w[i4].y, dot);
          dot = __fmaf_rn(tw.z, w[i4].z, dot);
          dot = __fmaf_rn(tw.w, w[i4].w, dot);
          nj = __fmaf_rn(w[i4].x, w[i4].x, nj);
          nj = __fmaf_rn(w[i4].y, w[i4].y, nj);
          nj = __fmaf_rn(w[i4].z, w[i4].z, nj);
          nj = __fmaf_rn(w[i4].w, w[i4].w, nj);
        }
        const float dist = __fadd_rn(__fadd_rn(__fsub_rn(sm.norms[rr], dot), nj), 0.0f);
        atomicMin(&sm.best[rr],
                  (static_cast<unsigned long long>(order_key(dist)) << 32) | static_cast<uint32_t>(j));
      }
      // every candidate of every row is in; is any row flagged?
      const int any_slow = epi_bar_or(slow_flag);
      int winner = -1;
      if (owner && fast && sm.row_bad[lr] == 0 && sm.best[lr] != ~0ull)
        winner = static_cast<int>(sm.best[lr] & 0xffffffffu);
      int nslow = 0;
      if (any_slow) {
        if (owner && valid && winner < 0) {
          const int at = atomicAdd(&sm.slow_count, 1);
          sm.slow_list[at] = lr;
        }
        epi_bar();
        nslow = sm.slow_count;
      }
      if (nslow > 0) {
        // exact scan, one warp per row; 2r is read back from the A image
        for (int i = warp; i < nslow; i += kEpiThreads / 32) {
          const int sr = sm.slow_list[i];
          float tw[kDim];
          for (int d = 0; d < kDim; ++d)
            tw[d] = *reinterpret_cast<const float*>(a_bytes + sw128_offset(sr, d, kRows * 128u));
          const int ix = exact_scan(tw, sm.norms[sr], book, cnorm, a.k, lane);
          if (lane == 0) sm.sel[sr] = ix;
        }
        epi_bar();
        if (owner && valid && winner < 0) winner = sm.sel[lr];
        epi_bar();
        if (warp == 0 && lane == 0) sm.slow_count = 0;
      }
      // ---- update the residual (the reconstruction is summed at the end).
      // A row's code is the exact scan's where it took one, else the key
      // minimum; both are final here, so every thread updates its own units.
#pragma unroll
      for (int i = 0; i < kUnits; ++i) {
        if (!unit_valid(i)) continue;
        const int row = unit_row(i);
        int w = sm.sel[row];
        if (w < 0) {
          const unsigned long long key = sm.best[row];
          if (key != ~0ull) {
            w = static_cast<int>(key & 0xffffffffu);
          } else {
            // Unreachable: on the fast path the screening maximum is a real
            // code (padding codes screen at -inf, real ones are finite), so
            // every row outside the exact scan has a resolved candidate.
            // Kept in bounds, reported.
            if (uchunk == 0) record_device_error(MOSS_ERR_UNSUPPORTED);
            w = 0;
          }
        }
        const float4 v =
            reinterpret_cast<const float4*>(book + static_cast<int64_t>(w) * kDim)[uchunk];
        r4[i].x = __fsub_rn(r4[i].x, v.x);
        r4[i].y = __fsub_rn(r4[i].y, v.y);
        r4[i].z = __fsub_rn(r4[i].z, v.z);
        r4[i].w = __fsub_rn(r4[i].w, v.w);
        if (uchunk == 0) a.codes[static_cast<int64_t>(s) * a.rows + row0 + row] = w;
      }
      // every reader of this stage's A image (MMA, exact distances, slow
      // scan) is done: the next stage's operand can go in
      if (s + 1 < a.stages) write_a();
      // the slow scan read the A image and the resolve read the other parts'
      // records: both must be finished before the next stage rewrites them
      epi_bar();
    }
    if (!aborted) {
      // recon = sum of the chosen codewords in stage order from +0 (the same
      // float32 additions as an incremental sum), unit by unit.  The codes
      // were stored by the rows' first-unit threads before the stage
      // barriers; they are read past L1.
      float4 acc[kUnits];
#pragma unroll
      for (int i = 0; i < kUnits; ++i) acc[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      for (int s = 0; s < a.stages; ++s) {
#pragma unroll
        for (int i = 0; i < kUnits; ++i) {
          if (!unit_valid(i)) continue;
          const int c = __ldcg(a.codes + static_cast<int64_t>(s) * a.rows + row0 + unit_row(i));
          const float4 v = reinterpret_cast<const float4*>(
              a.books + (static_cast<int64_t>(s) * a.k + c) * kDim)[uchunk];
          acc[i].x = __fadd_rn(acc[i].x, v.x);
          acc[i].y = __fadd_rn(acc[i].y, v.y);
          acc[i].z = __fadd_rn(acc[i].z, v.z);
          acc[i].w = __fadd_rn(acc[i].w, v.w);
        }
      }
#pragma unroll
      for (int i = 0; i < kUnits; ++i) {
        if (!unit_valid(i)) continue;
        const int64_t g = row0 + unit_row(i);
        reinterpret_cast<float4*>(a.recon + g * kDim)[uchunk] = acc[i];
        if (a.residual_out) reinterpret_cast<float4*>(a.residual_out + g * kDim)[uchunk] = r4[i];
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}

}  // namespace rvqtc
}  // namespace moss

using namespace moss;

namespace moss {
int rvq_pair_capacity(size_t smem);
size_t rvq_pair_smem();
int launch_rvq_pair(const rvqtc::Args& args, int64_t pairs, void* stream);
}  // namespace moss

extern "C" int moss_rvq_encode_kernel(const float* x, int64_t rows, int64_t d, const float* books,
                                      const float* packed, const float* code_norm,
                                      const float* stats, int64_t stages, int64_t k,
                                      int32_t* codes, float* recon, float* residual_out,
                                      int kernel, void* stream) {
  const char* name = "moss_rvq_encode";
  if (rows < 0 || stages < 1 || k < 1) return fail(MOSS_ERR_VALUE, "%s: bad shape", name);
  if (kernel != MOSS_RVQ_AUTO && kernel != MOSS_RVQ_SINGLE && kernel != MOSS_RVQ_PAIR)
    return fail(MOSS_ERR_VALUE, "%s: unknown kernel %d", name, kernel);
  if (d != rvqtc::kDim) return fail(MOSS_ERR_UNSUPPORTED, "%s: only 64-dim codewords are supported", name);
  if (k > rvqtc::kMaxCodes || stages > 65535)
    return fail(MOSS_ERR_UNSUPPORTED, "%s: at most 4096 codes per stage (use moss_rvq_encode_ffma)", name);
  if (rows == 0) return MOSS_OK;
  if (!x || !books || !packed || !code_norm || !stats || !codes || !recon)
    return fail(MOSS_ERR_VALUE, "%s: null pointer", name);
  if (!aligned16(x) || !aligned16(books) || !aligned16(packed) || !aligned16(code_norm) ||
      !aligned16(recon) || (residual_out && !aligned16(residual_out)))
    return fail(MOSS_ERR_VALUE, "%s: buffers must be 16-byte aligned", name);
  const int64_t kpad = (k + rvqtc::kTileCodes - 1) / rvqtc::kTileCodes * rvqtc::kTileCodes;
  const int64_t sms = sm_count();
  // The tensor-core tile images follow the FFMA layout in the packed buffer.
  const float* image = packed + stages * kpad * rvqtc::kDim;
  rvqtc::Args args{x, books, image, code_norm, stats, codes, recon, residual_out, rows,
                   static_cast<int>(stages), static_cast<int>(k), static_cast<int>(kpad), 0};

  // CTA pairs (rvq_pair.cu) on request, where the codebook has at least two
  // 256-code tiles and the rows fit one wave of pairs at <= 128 rows each:
  // the rows are spread evenly over the pairs that fit on the device at once
  // (8192 rows on 148 SMs -> 74 pairs of 111).  MOSS_RVQ_AUTO takes the
  // single-CTA kernel, the faster of the two as measured at 8192 x 32 x 1024.
  if (kernel == MOSS_RVQ_PAIR) {
    const int64_t ntiles = kpad / rvqtc::kTileCodes;
    int64_t pairs_max = ntiles >= 2 ? rvq_pair_capacity(rvq_pair_smem()) : 0;
    if (pairs_max > sms / 2) pairs_max = sms / 2;
    if (pairs_max >= 1 && rows <= pairs_max * rvqtc::kRows) {
      const int64_t per_pair = (rows + pairs_max - 1) / pairs_max;
      args.rows_per_cta = static_cast<int>(per_pair);
      return launch_rvq_pair(args, (rows + per_pair - 1) / per_pair, stream);
    }
    return fail(MOSS_ERR_UNSUPPORTED,
                  "%s: the pair kernel needs at least 257 codes and at most 128 rows per pair "
                  "(%lld pairs fit on this device)",
                  name, static_cast<long long>(pairs_max));
  }

  // One CTA per row block, the whole codebook each: while the rows fit one
  // CTA per SM at 64 rows per CTA, they are spread evenly over all SMs
  // (ceil(rows / SMs) rows per CTA, each row in two TMEM lanes so four
  // threads share its columns); above that a CTA takes 128 rows, one lane
  // each.
  const int rows_per_cta =
      rows <= sms * 64 ? static_cast<int>((rows + sms - 1) / sms) : rvqtc::kRows;
  const int64_t grid = (rows + rows_per_cta - 1) / rows_per_cta;
  if (grid > 0x7fffffffLL) return fail(MOSS_ERR_UNSUPPORTED, "%s: too many rows", name);
  args.rows_per_cta = rows_per_cta;
  const size_t smem = sizeof(rvqtc::Smem) + 1024;
  static bool configured[kMaxDevices] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices || !configured[dev]) {
    for (auto fn : {rvqtc::rvq_tc_kernel<1>, rvqtc::rvq_tc_kernel<2>}) {
      cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
      if (e != cudaSuccess) return fail(MOSS_ERR_CUDA, "%s: %s", name, cudaGetErrorString(e));
    }
    if (dev >= 0 && dev < kMaxDevices) configured[dev] = true;
  }
  const dim3 blocks(static_cast<unsigned>(grid));
  if (rows_per_cta <= rvqtc::kRows / 2)
    rvqtc::rvq_tc_kernel<2><<<blocks, rvqtc::kThreads, smem, as_stream(stream)>>>(args);
  else
    rvqtc::rvq_tc_kernel<1><<<blocks, rvqtc::kThreads, smem, as_stream(stream)>>>(args);
  return launch_status(name);
}

extern "C" int moss_rvq_encode(const float* x, int64_t rows, int64_t d, const float* books,
                               const float* packed, const float* code_norm, const float* stats,
                               int64_t stages, int64_t k, int32_t* codes, float* recon,
                               float* residual_out, void* stream) {
  return moss_rvq_encode_kernel(x, rows, d, books, packed, code_norm, stats, stages, k, codes,
                                recon, residual_out, MOSS_RVQ_AUTO, stream);
}
