// Persistent tensor-core triangular solve, op(A) X = B in place (bf16 A).
//
// The solve is cut into tasks (j, c): block row j (NB2 = 128 rows, in solve
// order) of column tile c (NC = 128 right-hand-side columns).  Left-looking:
//   D    = sum_{s solved before j} op(A)_{j,s} X_{s,c}   tcgen05, bf16 operands, fp32 TMEM
//   Y    = B_{j,c} - D                                    fp32
//   X_jc = inv(op(A)_{j,j}) Y                             tcgen05, 3-term bf16 split
// Columns are independent, so task (j, c) depends only on the tasks (s, c)
// before it in its column tile.  One CTA per SM takes tasks from a global
// ticket counter in level order (all tasks of block row 0, then of block row
// 1, ...), a topological order of the dependencies: a task waits only for
// tasks with lower tickets, which went to CTAs already running.  A finished
// task publishes its solved block as a bf16 operand image in global memory and
// raises a readiness flag; the tasks below it in the column tile bring that
// image in by bulk copy.  128 columns per task (against 32 per CTA in a
// column-owning layout) give each copied 32 KB tile of A four times the
// tensor-core work, and every SM has tasks even when the right-hand side is
// narrow.
// Warp roles (192 threads):
//   warps 0-3  epilogue: TMEM lanes 32w..32w+31 = rows of the block; the
//              right-hand side into the accumulator, Y, X_jc, the bf16 image
//              and its readiness flag, the writes of X
//   warp 4     producer: takes tickets, waits (bounded) for the flags of the
//              blocks a task needs, and issues the bulk copies of the packed
//              op(A)_{j,s} tile and of X_{s,c} (64 KB per stage, two stages),
//              then of the two inverse tiles inv(op(A)_jj) hi / lo
//   warp 5     MMA issue
// D is double-buffered in TMEM, so the next task's products start while this
// task's epilogue runs.  Before the solve, pack_tiles_kernel writes every
// strictly upper 128 x 128 block of A once as the shared-memory image of the
// operand tile it becomes (K-major for op = A, MN-major transposed for
// op = A^T) and clears the readiness flags; diag_inverse_layout_kernel writes
// the inverses of the diagonal blocks (fp32 column substitution, four threads
// per column, 3-term bf16 split) in the operand layout.
// Every wait is bounded: a role that gives up raises the launch's abort word,
// every role of every CTA stops at its next wait, and the launch reports
// IFK_ERR_TIMEOUT.
#include "ifk_common.cuh"
#include "ifk_internal.h"
#include "tc.cuh"

namespace ifk {

namespace {

constexpr int NB2 = 128;  // block rows of A (diagonal blocks)
constexpr int NC = 128;   // right-hand-side columns of a task (column tile)
constexpr int NSTAGE = 2;
constexpr int NTQ = 2;    // task queue slots (the task in flight and the next): tickets are not hoarded
constexpr int TPB = 192;
constexpr int MAXP = TRSM_MAX_PROBLEMS;
constexpr int MAXLVL = 256;  // block rows per problem (orders up to 32768)

constexpr uint32_t SZ_A = NB2 * NB2 * 2;  // 32 KB
constexpr uint32_t SZ_X = NB2 * NC * 2;   // 32 KB
constexpr uint32_t SZ_STAGE = SZ_A + SZ_X;
constexpr uint32_t OFF_YH = NSTAGE * SZ_STAGE;
constexpr uint32_t OFF_YL = OFF_YH + SZ_X;
constexpr uint32_t OFF_BAR = OFF_YL + SZ_X;
// barriers (8 bytes each)
enum {
  B_FULL = 0, B_EMPTY = NSTAGE, B_DFULL = 2 * NSTAGE, B_DINIT = B_DFULL + 2, B_YRDY = B_DINIT + 2,
  B_XFULL = B_YRDY + 1, B_XFREE = B_XFULL + 2, B_FIN = B_XFREE + 2, B_TFULL, B_TEMPTY = B_TFULL + NTQ,
  B_COUNT = B_TEMPTY + NTQ
};
constexpr uint32_t OFF_TASK = OFF_BAR + 8 * B_COUNT;  // NTQ task slots of 4 ints
constexpr uint32_t OFF_MISC = OFF_TASK + 16 * NTQ;    // TMEM slot
constexpr uint32_t SMEM = OFF_MISC + 16;
static_assert(SZ_STAGE % 1024 == 0 && OFF_YH % 1024 == 0, "bulk-copy destinations stay 1024-byte aligned");
static_assert(SMEM <= 227 * 1024, "shared memory of one CTA");

constexpr uint32_t A_MN = 128, A_K = (NB2 / 8) * 128;  // A tiles: core matrices 128 B apart along MN
constexpr uint32_t X_N = 128, X_K = (NC / 8) * 128;    // X / Y tiles (MN-major, mn = column)
// TMEM: D double-buffered (the next task's products run under this task's epilogue)
// and X double-buffered (the next task's diagonal solve runs while this task's X is
// written out)
constexpr uint32_t TM_D0 = 0, TM_D1 = NC, TM_X0 = 2 * NC, TM_X1 = 3 * NC, TM_COLS = 512;

#ifdef IFK_TRACE
// Diagnostic build only: per-task timestamps (globaltimer, ns) of the last solve
// launch, indexed by ticket: 0 CTA, 1 picked, 2 first copy issued, 3 last flag seen,
// 4 D ready, 5 Y ready, 6 X ready, 7 flag published, 8 end.
constexpr int TTR = 10;
__device__ long long g_trsm_trace[8192 * TTR];
__device__ __forceinline__ long long gtime_ns() {
  long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
#define TT_SET(tk, i, v) \
  if ((tk) < 8192) g_trsm_trace[(size_t)(tk) * TTR + (i)] = (v)
#else
#define TT_SET(tk, i, v)
#endif
constexpr size_t INV_SMEM = 2 * sizeof(float) * NB2 * (NB2 + 1);
// Every wait gives up after a few seconds: an mbarrier poll suspends for at most
// WAIT_HINT_NS, a flag poll is one load from L2.
constexpr uint32_t WAIT_LIMIT = 1u << 22;   // mbarrier polls
constexpr uint32_t WAIT_HINT_NS = 1000;     // suspend-time hint of one poll
constexpr uint32_t FLAG_LIMIT = 1u << 24;   // polls of another CTA's readiness flag (an L2 round trip each)

// One launch serves up to MAXP problems (the layers of a batched natural
// gradient); a block finds its problem by binary search over the prefix of the
// blocks each problem takes.
struct PackBatch {
  const __nv_bfloat16* A[MAXP];
  int64_t ldA[MAXP], n[MAXP];
  uint8_t* tiles[MAXP];
  int* flags[MAXP];  // readiness flags to clear (nflag[q] ints, the ticket counter first)
  int nflag[MAXP];
  int blk0[MAXP + 1];
  int np, trans;
};
struct InvBatch {
  const __nv_bfloat16* A[2 * MAXP];
  int64_t ld[2 * MAXP], n[2 * MAXP];
  uint8_t* inv[2 * MAXP];
  int blk0[2 * MAXP + 1];
  int nm;
};
struct SolveBatch {
  const uint8_t* tiles[MAXP];
  float* B[MAXP];
  int64_t rs[MAXP], cs[MAXP], n[MAXP], N[MAXP];
  const __nv_bfloat16* inv[MAXP];
  __nv_bfloat16* xws[MAXP];
  int* flags[MAXP];     // [nblk][ntile] readiness of solved blocks
  int nblk[MAXP], ntile[MAXP], vb[MAXP];
  int lvl_off[MAXLVL + 1];  // first ticket of each level (block row in solve order)
  int nlvl, ntasks, np, trans;
  int* ctr;             // ticket counter (the first word of problem 0's flags area)
  int* abort_;          // raised when a wait gave up (the second word)
  int* err;
};
// problem q with blk0[q] <= block < blk0[q + 1]
__device__ __forceinline__ int find_problem(const int* blk0, int np, int block) {
  int lo = 0, hi = np;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (blk0[mid] <= block) lo = mid;
    else hi = mid;
  }
  return lo;
}

__device__ __forceinline__ uint32_t bar_addr(uint32_t sb, int i) { return sb + OFF_BAR + 8u * (uint32_t)i; }

__device__ __forceinline__ void arrive_expect(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}
// Count `bytes` of an expected transfer as arrived (a copy that will not be issued).
__device__ __forceinline__ void complete_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.complete_tx.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void commit_to(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}
// Bounded wait on a barrier phase that also gives up once another role aborted.
__device__ __forceinline__ bool wait_phase(uint32_t bar, uint32_t parity, volatile int* abort_) {
  for (uint32_t it = 0; it < WAIT_LIMIT; ++it) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(bar), "r"(parity), "r"(WAIT_HINT_NS)
        : "memory");
    if (done) return true;
    if ((it & 255) == 255 && *abort_) return false;
  }
  *abort_ = 1;
  return false;
}
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
__device__ __forceinline__ void st16(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint4 pack8(const float* v) {
  return make_uint4(tc::pack_bf16(v[0], v[1]), tc::pack_bf16(v[2], v[3]), tc::pack_bf16(v[4], v[5]),
                    tc::pack_bf16(v[6], v[7]));
}

// Strictly upper block (a, b), a < b, of A as the image of an operand tile:
// op = A: tile op(A)_{a,b} = A_ab, K-major (mn = row, k = column);
// op = A^T: tile op(A)_{b,a} = A_ab^T, MN-major (mn = column, k = row).
// Tile index b (b - 1) / 2 + a; one CTA per tile, staged through shared memory
// so both the reads of A and the writes of the image are contiguous.
// Blocks past the tiles clear the readiness flags of one problem each.
__global__ void __launch_bounds__(256) pack_tiles_kernel(const __grid_constant__ PackBatch pb) {
  extern __shared__ __align__(16) uint8_t img[];
  if ((int)blockIdx.x >= pb.blk0[pb.np]) {
    const int q = (int)blockIdx.x - pb.blk0[pb.np];
    for (int i = threadIdx.x; i < pb.nflag[q]; i += 256) pb.flags[q][i] = 0;
    return;
  }
  const int q = find_problem(pb.blk0, pb.np, (int)blockIdx.x);
  const __nv_bfloat16* A = pb.A[q];
  const int64_t ldA_ = pb.ldA[q], n = pb.n[q];
  const int trans = pb.trans;
  uint8_t* tiles = pb.tiles[q];
  const int t = (int)blockIdx.x - pb.blk0[q];
  int b = (int)((1.0 + sqrt(1.0 + 8.0 * t)) * 0.5);
  while (b * (b - 1) / 2 > t) --b;
  while ((b + 1) * b / 2 <= t) ++b;
  const int a = t - b * (b - 1) / 2;
  const int64_t a0 = (int64_t)a * NB2, b0 = (int64_t)b * NB2;
  for (int it = threadIdx.x; it < NB2 * (NB2 / 8); it += 256) {
    const int i = it >> 4, c = it & 15;  // row i of the block, 16-byte chunk c (columns 8c .. 8c + 7)
    uint4 v = make_uint4(0, 0, 0, 0);
    if (a0 + i < n && b0 + 8 * c < n) v = *reinterpret_cast<const uint4*>(A + (a0 + i) * ldA_ + b0 + 8 * c);
    const uint32_t off = trans ? (uint32_t)(i >> 3) * A_K + (uint32_t)c * A_MN + (uint32_t)(i & 7) * 16u
                               : (uint32_t)c * A_K + (uint32_t)(i >> 3) * A_MN + (uint32_t)(i & 7) * 16u;
    *reinterpret_cast<uint4*>(img + off) = v;
  }
  __syncthreads();
  uint4* dst = reinterpret_cast<uint4*>(tiles + (size_t)t * SZ_A);
  for (int it = threadIdx.x; it < (int)(SZ_A / 16); it += 256) dst[it] = reinterpret_cast<const uint4*>(img)[it];
}

// inv(A_bb) of the upper-triangular diagonal blocks (fp32 column substitution),
// written as bf16 hi / lo in both operand layouts: the K-major tile of inv(A_bb)
// (op = A) and the MN-major tile of its transpose (op = A^T).  Block b of matrix
// m in [hi K, lo K, hi MN, lo MN] order (SZ_A each) at inv_m + b * 4 * SZ_A.
// One launch covers every block of a list of matrices.  Ragged last block:
// identity pad.
constexpr int INV_TPB = 4 * NB2;  // four threads per column of the inverse
__global__ void __launch_bounds__(INV_TPB) diag_inverse_layout_kernel(const __grid_constant__ InvBatch ib) {
  extern __shared__ float dsm[];
  float (*U)[NB2 + 1] = reinterpret_cast<float (*)[NB2 + 1]>(dsm);
  float (*Xs)[NB2 + 1] = reinterpret_cast<float (*)[NB2 + 1]>(dsm + NB2 * (NB2 + 1));
  const int mat = find_problem(ib.blk0, ib.nm, (int)blockIdx.x);
  const __nv_bfloat16* A = ib.A[mat];
  const int64_t ldA_ = ib.ld[mat], n = ib.n[mat];
  const int b = (int)blockIdx.x - ib.blk0[mat], t = threadIdx.x;
  const int64_t b0 = (int64_t)b * NB2;
  const int nb = (int)mn<int64_t>(NB2, n - b0);
  for (int idx = t; idx < NB2 * NB2; idx += INV_TPB) {
    const int r = idx / NB2, l = idx % NB2;
    float v = (r == l) ? 1.f : 0.f;
    if (r < nb && l < nb) v = (l >= r) ? __bfloat162float(A[(b0 + r) * ldA_ + b0 + l]) : 0.f;
    U[r][l] = v;
  }
  __syncthreads();
  // Column q of U^-1 by column-oriented back substitution: the four lanes of a
  // column (one warp quad) hold the residues of its rows l = 4k + part in
  // registers; once x_r = res_r / U[r][r] is known (a shuffle from the lane of
  // row r), every lane folds it into the residues of its rows above r.  A step
  // is one shuffle, one divide and independent FMAs, so the chain from row r to
  // row r - 1 is short; the U[l][r] reads of a warp hit four consecutive banks.
  {
    const int q = t >> 2, part = t & 3, lane = t & 31;
    float res[NB2 / 4];
#pragma unroll
    for (int k = 0; k < NB2 / 4; ++k) res[k] = (4 * k + part == q) ? 1.f : 0.f;
#pragma unroll
    for (int r = NB2 - 1; r >= 0; --r) {
      const float x = __shfl_sync(0xffffffffu, res[r >> 2], (lane & ~3) | (r & 3)) / U[r][r];
      if (part == (r & 3)) Xs[r][q] = x;
#pragma unroll
      for (int k = 0; k <= (r >> 2); ++k)
        if (4 * k + part < r) res[k] = fmaf(-U[4 * k + part][r], x, res[k]);
    }
  }
  __syncthreads();
  uint8_t* o = ib.inv[mat] + (size_t)b * 4 * SZ_A;
  for (int it = t; it < NB2 * (NB2 / 8); it += INV_TPB) {
    // K-major: 8 consecutive k = l of row m; MN-major (transpose): 8 consecutive mn = l of k = m
    const int m = it >> 4, l8 = it & 15;
    float hi[8], lo[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) tc::split_bf16(Xs[m][l8 * 8 + e], hi[e], lo[e]);
    const uint32_t offk = (uint32_t)l8 * A_K + (uint32_t)(m >> 3) * A_MN + (uint32_t)(m & 7) * 16u;
    const uint32_t offm = (uint32_t)(m >> 3) * A_K + (uint32_t)l8 * A_MN + (uint32_t)(m & 7) * 16u;
    const uint4 vh = pack8(hi), vl = pack8(lo);
    *reinterpret_cast<uint4*>(o + offk) = vh;
    *reinterpret_cast<uint4*>(o + SZ_A + offk) = vl;
    *reinterpret_cast<uint4*>(o + 2 * SZ_A + offm) = vh;
    *reinterpret_cast<uint4*>(o + 3 * SZ_A + offm) = vl;
  }
}

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release(int* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Bounded wait for another CTA's readiness flag; gives up early once the launch aborted.
__device__ __forceinline__ bool wait_flag(const int* f, volatile int* abort_) {
  for (uint32_t it = 0; it < FLAG_LIMIT; ++it) {
    if (ld_acquire(f) != 0) return true;
    if ((it & 31) == 31 && *abort_) return false;
  }
  *abort_ = 1;
  return false;
}
// Bounded wait that ignores the abort word: used before exit, for copies and MMAs
// already in flight, which complete whatever the other roles do.
__device__ __forceinline__ bool drain_phase(uint32_t bar, uint32_t parity) {
  for (uint32_t it = 0; it < WAIT_LIMIT; ++it) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(bar), "r"(parity), "r"(WAIT_HINT_NS)
        : "memory");
    if (done) return true;
  }
  return false;
}

static_assert(sizeof(SolveBatch) <= 32000, "launch parameters of one solve launch (limit 32764 bytes)");
static_assert(sizeof(PackBatch) <= 32000, "launch parameters of one pack launch");

// ticket -> (problem, level = block row in solve order, column tile); level-major,
// then problem, then column tile
__device__ __forceinline__ void decode_task(const SolveBatch& b, int tk, int* q, int* lvl, int* c) {
  int lo = 0, hi = b.nlvl;  // lvl_off[lo] <= tk < lvl_off[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (b.lvl_off[mid] <= tk) lo = mid;
    else hi = mid;
  }
  int r = tk - b.lvl_off[lo];
  for (int p = 0; p < b.np; ++p) {
    if (b.nblk[p] <= lo) continue;
    if (r < b.ntile[p]) {
      *q = p;
      *lvl = lo;
      *c = r;
      return;
    }
    r -= b.ntile[p];
  }
  *q = -1;
}

__global__ void __launch_bounds__(TPB, 1) trsm_persist_kernel(const __grid_constant__ SolveBatch sbt) {
  extern __shared__ __align__(1024) uint8_t sm[];
  const uint32_t sb = tc::smem_u32(sm);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + OFF_MISC);
  int4* tq = reinterpret_cast<int4*>(sm + OFF_TASK);
  volatile int* abort_ = sbt.abort_;
  int* err = sbt.err;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int trans = sbt.trans;
  auto bar = [&](int i) { return bar_addr(sb, i); };

  if (warp == 0) tc::tmem_alloc(tslot, TM_COLS);
  if (tid == 0) {
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
    for (int i = 0; i < NSTAGE; ++i) {
      tc::mbar_init(bars + B_FULL + i, 1);
      tc::mbar_init(bars + B_EMPTY + i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(bars + B_DFULL + i, 1);
      tc::mbar_init(bars + B_DINIT + i, 4);
    }
    tc::mbar_init(bars + B_YRDY, 4);
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(bars + B_XFULL + i, 1);
      tc::mbar_init(bars + B_XFREE + i, 4);
    }
    tc::mbar_init(bars + B_FIN, 1);
    for (int i = 0; i < NTQ; ++i) {
      tc::mbar_init(bars + B_TFULL + i, 1);
      tc::mbar_init(bars + B_TEMPTY + i, 5);
    }
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tm = *tslot;

  if (warp == 4) {
    // ---------------- producer: tickets, readiness flags, bulk copies ----------------
    // Lane 0 takes the tickets and issues the copies; the whole warp brings each new
    // task's right-hand side into L2 first, so the epilogue's loads of it are L2 hits.
    uint32_t g = 0;  // stage fills issued (lane 0)
    bool ok = true;
    for (int k = 0;; ++k) {
      const int slot = k % NTQ;
      int q = -1, lvl = 0, c = 0, tk = 0;
      if (lane == 0) {
        if (k >= NTQ) ok = wait_phase(bar(B_TEMPTY + slot), ((k / NTQ) - 1) & 1, abort_);
        if (ok && !*abort_) {
          tk = atomicAdd(sbt.ctr, 1);
          if (tk < sbt.ntasks) decode_task(sbt, tk, &q, &lvl, &c);
        }
        tq[slot] = make_int4(q, lvl, c, tk);
        TT_SET(tk, 0, (long long)blockIdx.x);
        TT_SET(tk, 1, gtime_ns());
        arrive(bar(B_TFULL + slot));  // q < 0 tells the other roles to stop
      }
      q = __shfl_sync(0xffffffffu, q, 0);
      lvl = __shfl_sync(0xffffffffu, lvl, 0);
      c = __shfl_sync(0xffffffffu, c, 0);
      if (q < 0) break;
      const int nb = sbt.nblk[q], nt = sbt.ntile[q];
      const int jb = trans ? lvl : nb - 1 - lvl;
      {
        const int64_t j0 = (int64_t)jb * NB2, c0 = (int64_t)c * NC, rs = sbt.rs[q], cs = sbt.cs[q];
        const int nj = (int)mn<int64_t>(NB2, sbt.n[q] - j0), nc = (int)mn<int64_t>(NC, sbt.N[q] - c0);
        // contiguous 512-byte lines of the tile: rows when columns are contiguous, else columns
        const bool by_row = cs == 1;
        const int nline = by_row ? nj : (rs == 1 ? nc : 0);
        const int len = by_row ? nc : nj;
        for (int li = lane; li < nline; li += 32) {
          const int64_t off = by_row ? (j0 + li) * rs + c0 : (c0 + li) * cs + j0;
          for (int e = 0; e < len; e += 32) prefetch_l2(sbt.B[q] + off + e);
        }
      }
      if (lane == 0) {
        const uint8_t* tiles = sbt.tiles[q];
        const uint8_t* xw = reinterpret_cast<const uint8_t*>(sbt.xws[q]);
        const int* flags = sbt.flags[q];
        // solved blocks of this column tile, oldest first (the newest is the one
        // most likely still in flight)
        for (int i = 0; i < lvl && ok; ++i) {
          const int s = trans ? i : nb - 1 - i;
          const int st = (int)(g % NSTAGE);
          if (g >= NSTAGE) ok = wait_phase(bar(B_EMPTY + st), ((g / NSTAGE) - 1) & 1, abort_);
          if (!ok) break;
          const uint32_t full = bar(B_FULL + st);
          const uint32_t dst = sb + (uint32_t)st * SZ_STAGE;
          arrive_expect(full, SZ_STAGE);
          // op(A)_{j,s} is the packed image of A block (min, max) of (j, s); it does not
          // depend on the flag, so its copy runs while the flag is awaited
          const int ta = jb < s ? jb : s, tb = jb < s ? s : jb;
          bulk_load(dst, tiles + (size_t)(tb * (tb - 1) / 2 + ta) * SZ_A, SZ_A, full);
          if (i == 0) TT_SET(tk, 2, gtime_ns());
          ok = wait_flag(flags + (size_t)s * nt + c, abort_);
          if (i == lvl - 1) TT_SET(tk, 3, gtime_ns());
          if (!ok) {
            // the X part never comes: account for its bytes, so the phase completes when the
            // A copy lands and the cleanup below can wait for that copy
            complete_tx(full, SZ_X);
            ++g;
            break;
          }
          asm volatile("fence.proxy.async.global;" ::: "memory");
          bulk_load(dst + SZ_A, xw + ((size_t)c * nb + s) * SZ_X, SZ_X, full);
          ++g;
        }
        // the inverse of the diagonal block, hi then lo, in the operand layout of op
        const uint8_t* src = reinterpret_cast<const uint8_t*>(sbt.inv[q]) + (size_t)jb * 4 * SZ_A +
                             (trans ? 2 * SZ_A : 0);
        for (int h = 0; h < 2 && ok; ++h) {
          const int st = (int)(g % NSTAGE);
          if (g >= NSTAGE) ok = wait_phase(bar(B_EMPTY + st), ((g / NSTAGE) - 1) & 1, abort_);
          if (!ok) break;
          arrive_expect(bar(B_FULL + st), SZ_A);
          bulk_load(sb + (uint32_t)st * SZ_STAGE, src + h * SZ_A, SZ_A, bar(B_FULL + st));
          ++g;
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
    }
    if (lane == 0 && !ok) {
      // copies already issued land whatever the consumers do: wait for them (bounded)
      for (uint32_t i = g > NSTAGE ? g - NSTAGE : 0; i < g; ++i)
        drain_phase(bar(B_FULL + (int)(i % NSTAGE)), (i / NSTAGE) & 1);
      *abort_ = 1;
      if (err) atomicExch(err, IFK_ERR_TIMEOUT);
    }
  } else if (warp == 5) {
    // ---------------- MMA issue ----------------
    if (lane == 0) {
      uint32_t g = 0;
      bool ok = true;
      const uint32_t idK = tc::idesc_bf16(128, NC, trans != 0, true);
      const uint32_t idKneg = idK | (1u << 13);  // D -= A X: the negate-A bit
      for (int k = 0;; ++k) {
        const int slot = k % NTQ;
        ok = wait_phase(bar(B_TFULL + slot), (k / NTQ) & 1, abort_);
        if (!ok) break;
        const int4 t = tq[slot];
        if (t.x < 0) break;
        const int lvl = t.y, db = k & 1;
        const uint32_t dcol = db ? TM_D1 : TM_D0, xcol = db ? TM_X1 : TM_X0;
        // D holds the right-hand side block (written by the epilogue, which has read
        // this buffer's previous contents); the products are subtracted from it
        ok = wait_phase(bar(B_DINIT + db), (k >> 1) & 1, abort_);
        if (!ok) break;
        tc::fence_after();
        for (int i = 0; i < lvl && ok; ++i) {
          const int st = (int)(g % NSTAGE);
          ok = wait_phase(bar(B_FULL + st), (g / NSTAGE) & 1, abort_);
          if (!ok) break;
          tc::fence_after();
          const uint32_t a0 = sb + (uint32_t)st * SZ_STAGE, x0 = a0 + SZ_A;
          const uint64_t ad = tc::sdesc(a0, A_K, A_MN), bd = tc::sdesc(x0, X_K, X_N);
#pragma unroll
          for (int kk = 0; kk < NB2 / 16; ++kk)
            tc::mma_bf16(tm + dcol, ad + tc::doff(kk * 2 * A_K), bd + tc::doff(kk * 2 * X_K), idKneg, 1u);
          commit_to(bar(B_EMPTY + st));
          ++g;
        }
        if (!ok) break;
        commit_to(bar(B_DFULL + db));
        // X = inv_hi Y_hi + inv_hi Y_lo + inv_lo Y_hi (the inverse tiles in the next two stages)
        const int sh = (int)(g % NSTAGE), sl = (int)((g + 1) % NSTAGE);
        ok = wait_phase(bar(B_FULL + sh), (g / NSTAGE) & 1, abort_) &&
             wait_phase(bar(B_FULL + sl), ((g + 1) / NSTAGE) & 1, abort_) &&
             wait_phase(bar(B_YRDY), k & 1, abort_) &&
             (k < 2 || wait_phase(bar(B_XFREE + db), ((k >> 1) - 1) & 1, abort_));
        if (!ok) break;
        tc::fence_after();
        {
          const uint64_t ah = tc::sdesc(sb + (uint32_t)sh * SZ_STAGE, A_K, A_MN);
          const uint64_t al = tc::sdesc(sb + (uint32_t)sl * SZ_STAGE, A_K, A_MN);
          const uint64_t yh = tc::sdesc(sb + OFF_YH, X_K, X_N), yl = tc::sdesc(sb + OFF_YL, X_K, X_N);
#pragma unroll
          for (int kk = 0; kk < NB2 / 16; ++kk) {
            const uint64_t da = tc::doff(kk * 2 * A_K), dx = tc::doff(kk * 2 * X_K);
            tc::mma_bf16(tm + xcol, ah + da, yh + dx, idK, kk > 0);
            tc::mma_bf16(tm + xcol, ah + da, yl + dx, idK, 1);
            tc::mma_bf16(tm + xcol, al + da, yh + dx, idK, 1);
          }
        }
        commit_to(bar(B_EMPTY + sh));
        commit_to(bar(B_EMPTY + sl));
        commit_to(bar(B_XFULL + db));
        g += 2;
        arrive(bar(B_TEMPTY + slot));
      }
      // every MMA issued has completed before the CTA releases TMEM
      commit_to(bar(B_FIN));
      drain_phase(bar(B_FIN), 0);
      if (!ok) {
        *abort_ = 1;
        if (err) atomicExch(err, IFK_ERR_TIMEOUT);
      }
    }
  } else {
    // ---------------- epilogue: warps 0-3, thread r = row of the block ----------------
    const int r = tid;
    const uint32_t lane_base = tm + ((uint32_t)(warp * 32) << 16);
    bool ok = true;
    // geometry of a task
    struct Geo {
      int q, lvl, c, nb, jb, nj, nc, tkn;
      int64_t j0, c0, rs, cs;
      float* B;
      bool vec;
    };
    auto geo = [&](const int4& t) {
      Geo G;
      G.q = t.x;
      G.lvl = t.y;
      G.c = t.z;
      G.tkn = t.w;
      G.nb = sbt.nblk[G.q];
      G.jb = trans ? G.lvl : G.nb - 1 - G.lvl;
      G.B = sbt.B[G.q];
      G.rs = sbt.rs[G.q];
      G.cs = sbt.cs[G.q];
      G.j0 = (int64_t)G.jb * NB2;
      G.c0 = (int64_t)G.c * NC;
      G.nj = (int)mn<int64_t>(NB2, sbt.n[G.q] - G.j0);
      G.nc = (int)mn<int64_t>(NC, sbt.N[G.q] - G.c0);
      G.vec = G.cs == 1 && sbt.vb[G.q];
      return G;
    };
    // The right-hand side block B_jc into the task's D buffer (row r of the block in
    // TMEM lane r), then DINIT: the products are subtracted from it, so D ends as
    // Y = B_jc - sum op(A)_{j,s} X_s with no global load between the last product and
    // the diagonal solve (the producer brought B_jc into L2 when it took the ticket).
    auto init_d = [&](const Geo& G, int dbuf) {
      const uint32_t dcol = dbuf ? TM_D1 : TM_D0;
#pragma unroll 2
      for (int g4 = 0; g4 < NC / 32; ++g4) {
        const int cv = G.nc - g4 * 32;  // valid columns of this group
        float bv[32];
        if (G.vec) {
#pragma unroll
          for (int g = 0; g < 8; ++g) {
            const float4 x = r < G.nj ? ld4(G.B + (G.j0 + r) * G.rs + G.c0 + g4 * 32 + 4 * g, cv - 4 * g)
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
            bv[4 * g] = x.x;
            bv[4 * g + 1] = x.y;
            bv[4 * g + 2] = x.z;
            bv[4 * g + 3] = x.w;
          }
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            bv[e] = (r < G.nj && e < cv) ? G.B[(G.j0 + r) * G.rs + (G.c0 + g4 * 32 + e) * G.cs] : 0.f;
        }
        tc::tmem_st32(lane_base + dcol + g4 * 32, bv);
      }
      tc::tmem_st_wait();
      tc::fence_before();
      __syncwarp();
      if (lane == 0) arrive(bar(B_DINIT + dbuf));
    };
    bool pre = false;  // D of this task was written during the previous one
    for (int k = 0;; ++k) {
      const int slot = k % NTQ;
      ok = wait_phase(bar(B_TFULL + slot), (k / NTQ) & 1, abort_);
      if (!ok) break;
      const int4 t = tq[slot];
      if (t.x < 0) break;
      const Geo G = geo(t);
      const int db = k & 1;
      const int tkn = G.tkn;
      (void)tkn;
      if (!pre) init_d(G, db);
      pre = false;
      ok = wait_phase(bar(B_DFULL + db), (k >> 1) & 1, abort_);
      if (!ok) break;
      tc::fence_after();
      TT_SET(tkn, 4, gtime_ns());
      // Y = D as bf16 hi / lo operand images, 32 columns at a time
#pragma unroll 1
      for (int g4 = 0; g4 < NC / 32; ++g4) {
        float y[32];
        tc::tmem_ld32(lane_base + (db ? TM_D1 : TM_D0) + g4 * 32, y);
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          float hi[8], lo[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) tc::split_bf16(y[g * 8 + e], hi[e], lo[e]);
          const uint32_t off = tc::cm_off<false>(g4 * 32 + g * 8, r, X_N, X_K);
          st16(sb + OFF_YH + off, pack8(hi));
          st16(sb + OFF_YL + off, pack8(lo));
        }
      }
      tc::fence_before();
      tc::fence_async_smem();
      __syncwarp();
      if (lane == 0) arrive(bar(B_YRDY));
      TT_SET(tkn, 5, gtime_ns());
      ok = wait_phase(bar(B_XFULL + db), (k >> 1) & 1, abort_);
      if (!ok) break;
      tc::fence_after();
      TT_SET(tkn, 6, gtime_ns());
      const uint32_t xcol = db ? TM_X1 : TM_X0;
      // First the bf16 image of X_jc for the tasks below it in this column tile (rows
      // past n and columns past N are exact zeros: their Y is zero), released behind
      // the readiness flag at once: the writes of X itself are off the chain.
      uint8_t* xo = reinterpret_cast<uint8_t*>(sbt.xws[G.q]) + ((size_t)G.c * G.nb + G.jb) * SZ_X;
#pragma unroll 1
      for (int g4 = 0; g4 < NC / 32; ++g4) {
        float x[32];
        tc::tmem_ld32(lane_base + xcol + g4 * 32, x);
#pragma unroll
        for (int g = 0; g < 4; ++g)
          *reinterpret_cast<uint4*>(xo + tc::cm_off<false>(g4 * 32 + g * 8, r, X_N, X_K)) = pack8(x + g * 8);
      }
      asm volatile("fence.proxy.async.global;" ::: "memory");
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (tid == 0) st_release(sbt.flags[G.q] + (size_t)G.jb * sbt.ntile[G.q] + G.c, 1);
      TT_SET(tkn, 7, gtime_ns());
      // the next task's right-hand side goes into its D buffer now, so its products
      // can start while this task's X is written out
      {
        const int slot1 = (k + 1) % NTQ;
        ok = wait_phase(bar(B_TFULL + slot1), ((k + 1) / NTQ) & 1, abort_);
        if (!ok) break;
        const int4 t1 = tq[slot1];
        if (t1.x >= 0) {
          init_d(geo(t1), db ^ 1);
          pre = true;
        }
      }
      const int64_t j0 = G.j0, c0 = G.c0, rs = G.rs, cs = G.cs;
      float* B = G.B;
#pragma unroll 1
      for (int g4 = 0; g4 < NC / 32; ++g4) {
        float x[32];
        tc::tmem_ld32(lane_base + xcol + g4 * 32, x);
        const int cv = G.nc - g4 * 32;
        if (r < G.nj) {
          if (G.vec) {
#pragma unroll
            for (int g = 0; g < 8; ++g)
              st4(B + (j0 + r) * rs + c0 + g4 * 32 + 4 * g,
                  make_float4(x[4 * g], x[4 * g + 1], x[4 * g + 2], x[4 * g + 3]), cv - 4 * g);
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (e < cv) B[(j0 + r) * rs + (c0 + g4 * 32 + e) * cs] = x[e];
          }
        }
      }
      tc::fence_before();
      __syncwarp();
      if (lane == 0) arrive(bar(B_XFREE + db));
      if (lane == 0) arrive(bar(B_TEMPTY + slot));
      TT_SET(tkn, 8, gtime_ns());
    }
    if (!ok) {
      *abort_ = 1;
      if (err) atomicExch(err, IFK_ERR_TIMEOUT);
    }
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after();
    tc::tmem_free(tm, TM_COLS);
  }
}

int sm_count() {
  static thread_local int dev_cached = -1, sms = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (dev != dev_cached) {
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    dev_cached = dev;
  }
  return sms;
}

bool attr_once() {
  static thread_local int done_dev = -1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  if (done_dev == dev) return true;
  if (cudaFuncSetAttribute(trsm_persist_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM) !=
      cudaSuccess)
    return false;
  if (cudaFuncSetAttribute(diag_inverse_layout_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)INV_SMEM) != cudaSuccess)
    return false;
  done_dev = dev;
  return true;
}

}  // namespace

#ifdef IFK_TRACE
extern "C" __attribute__((visibility("default"))) int ifk_trace_trsm_read(long long* dst, int max_tasks) {
  const int n = max_tasks < 8192 ? max_tasks : 8192;
  return cudaMemcpyFromSymbol(dst, g_trsm_trace, (size_t)n * TTR * sizeof(long long)) == cudaSuccess ? n : -1;
}
#endif

size_t trsm_persist_inverse_bytes(int64_t n) { return (size_t)cdiv(n, NB2) * 4 * SZ_A; }

// Scratch of one problem: bf16 images of the solved blocks [column tile][block row]
// | the control words (ticket counter, abort word) and readiness flags
// [block row][column tile] | the packed operand tiles of A.
namespace {
size_t xws_bytes(int64_t n, int64_t N) { return (size_t)cdiv(N, NC) * (size_t)cdiv(n, NB2) * SZ_X; }
constexpr int NCTRL = 16;  // control words before the flags
int nflags(int64_t n, int64_t N) { return NCTRL + (int)(cdiv(n, NB2) * cdiv(N, NC)); }
size_t flag_bytes(int64_t n, int64_t N) { return ((size_t)nflags(n, N) * 4 + 1023) / 1024 * 1024; }
}  // namespace

size_t trsm_persist_workspace(int64_t n, int64_t N) {
  const size_t nblk = (size_t)cdiv(n, NB2);
  return xws_bytes(n, N) + flag_bytes(n, N) + nblk * (nblk - 1) / 2 * SZ_A;
}

bool trsm_persist_ok(const void* A, int64_t ldA, int64_t n) {
  return ((uintptr_t)A % 16) == 0 && ldA % 8 == 0 && n % 8 == 0 && n >= 8;
}

int trsm_persist_prepare_many(int nm, const __nv_bfloat16* const* A, const int64_t* ld, const int64_t* n,
                              void* const* inv, cudaStream_t s) {
  if (!attr_once()) return IFK_ERR_CUDA;
  for (int base = 0; base < nm; base += 2 * MAXP) {
    InvBatch ib;
    ib.nm = nm - base < 2 * MAXP ? nm - base : 2 * MAXP;
    int acc = 0;
    for (int m = 0; m < ib.nm; ++m) {
      ib.A[m] = A[base + m];
      ib.ld[m] = ld[base + m];
      ib.n[m] = n[base + m];
      ib.inv[m] = (uint8_t*)inv[base + m];
      ib.blk0[m] = acc;
      acc += (int)cdiv(n[base + m], NB2);
    }
    ib.blk0[ib.nm] = acc;
    if (acc == 0) continue;
    diag_inverse_layout_kernel<<<(unsigned)acc, INV_TPB, INV_SMEM, s>>>(ib);
    IFK_CUDA_TRY(cudaGetLastError());
  }
  return IFK_OK;
}

int trsm_persist_prepare(const __nv_bfloat16* A0, int64_t ld0, int64_t n0, void* inv0, const __nv_bfloat16* A1,
                         int64_t ld1, int64_t n1, void* inv1, cudaStream_t s) {
  const __nv_bfloat16* A[2] = {A0, A1};
  const int64_t ld[2] = {ld0, ld1}, n[2] = {n0, n1};
  void* inv[2] = {inv0, inv1};
  return trsm_persist_prepare_many(A1 ? 2 : 1, A, ld, n, inv, s);
}

int trsm_persist_run_many(int np, const TrsmProblem* p, int trans, int* err, cudaStream_t s) {
  if (!attr_once()) return IFK_ERR_CUDA;
  const int sms = sm_count();
  if (sms <= 0) return IFK_ERR_CUDA;
  for (int base = 0; base < np; base += MAXP) {
    const int cnt = np - base < MAXP ? np - base : MAXP;
    PackBatch pb;
    SolveBatch sbt;
    pb.np = sbt.np = cnt;
    pb.trans = sbt.trans = trans;
    sbt.err = err;
    int tacc = 0, nlvl = 0;
    for (int q = 0; q < cnt; ++q) {
      const TrsmProblem& P = p[base + q];
      const int64_t nblk = cdiv(P.n, NB2);
      if (nblk > MAXLVL) return IFK_ERR_SHAPE;
      uint8_t* w = (uint8_t*)P.ws;
      __nv_bfloat16* xws = (__nv_bfloat16*)w;
      w += xws_bytes(P.n, P.N);
      int* flags = (int*)w;
      w += flag_bytes(P.n, P.N);
      pb.A[q] = P.A;
      pb.ldA[q] = P.ldA;
      pb.n[q] = P.n;
      pb.tiles[q] = w;
      pb.flags[q] = flags;
      pb.nflag[q] = nflags(P.n, P.N);
      pb.blk0[q] = tacc;
      tacc += (int)(nblk * (nblk - 1) / 2);
      sbt.tiles[q] = w;
      sbt.B[q] = P.B;
      sbt.rs[q] = P.rs;
      sbt.cs[q] = P.cs;
      sbt.n[q] = P.n;
      sbt.N[q] = P.N;
      sbt.inv[q] = (const __nv_bfloat16*)P.inv;
      sbt.xws[q] = xws;
      sbt.flags[q] = flags + NCTRL;
      sbt.nblk[q] = (int)nblk;
      sbt.ntile[q] = (int)cdiv(P.N, NC);
      // 16-byte vector access to rows of B needs 16-byte aligned rows
      sbt.vb[q] = (((uintptr_t)P.B % 16) == 0 && (P.rs * 4) % 16 == 0) ? 1 : 0;
      nlvl = nlvl > (int)nblk ? nlvl : (int)nblk;
    }
    pb.blk0[cnt] = tacc;
    // tickets in level order: every problem's column tiles of block row 0, then of 1, ...
    int acc = 0;
    for (int L = 0; L < nlvl; ++L) {
      sbt.lvl_off[L] = acc;
      for (int q = 0; q < cnt; ++q)
        if (sbt.nblk[q] > L) acc += sbt.ntile[q];
    }
    sbt.lvl_off[nlvl] = acc;
    sbt.nlvl = nlvl;
    sbt.ntasks = acc;
    sbt.ctr = pb.flags[0];
    sbt.abort_ = pb.flags[0] + 1;
    if (acc == 0) continue;
    // packs the tiles and clears the flags and control words (one block per problem)
    pack_tiles_kernel<<<(unsigned)(tacc + cnt), 256, SZ_A, s>>>(pb);
    IFK_CUDA_TRY(cudaGetLastError());
    trsm_persist_kernel<<<(unsigned)(acc < sms ? acc : sms), TPB, SMEM, s>>>(sbt);
    IFK_CUDA_TRY(cudaGetLastError());
  }
  return IFK_OK;
}

int trsm_persist_run(const __nv_bfloat16* A, int64_t ldA, int trans, float* B, int64_t rs, int64_t cs, int64_t n,
                     int64_t N, const void* inv, void* ws, int* err, cudaStream_t s) {
  const TrsmProblem p{A, ldA, B, rs, cs, n, N, inv, ws};
  return trsm_persist_run_many(1, &p, trans, err, s);
}

}  // namespace ifk
