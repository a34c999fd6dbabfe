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
//   warps 0-3  epilogue: TMEM lanes 32w..32w+31 = rows of the block; Y, X_jc,
//              the writes of X (or of the fused momentum / lr update) and of
//              the bf16 image, the readiness flag
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
// the inverses of the diagonal blocks (fp32 column substitution, 3-term bf16
// split) in the operand layout.
// Every wait is bounded: a role that gives up raises the launch's abort word,
// every role of every CTA stops at its next wait, and the launch reports
// IFK_ERR_TIMEOUT.
#include "ifk_common.cuh"
#include "ifk_internal.h"
#include "tc.cuh"

namespace ifk {

namespace {

constexpr int NB2 = 128;  // diagonal block
constexpr int NT = 32;    // right-hand-side columns per CTA
constexpr int NSTAGE = 3;
constexpr int TPB = 192;
constexpr int MAXP = TRSM_MAX_PROBLEMS;

constexpr uint32_t SZ_A = NB2 * NB2 * 2;  // 32 KB
constexpr uint32_t SZ_X = NB2 * NT * 2;   // 8 KB
constexpr uint32_t SZ_STAGE = SZ_A + SZ_X;
constexpr uint32_t OFF_IH = NSTAGE * SZ_STAGE;
constexpr uint32_t OFF_IL = OFF_IH + SZ_A;
constexpr uint32_t OFF_YH = OFF_IL + SZ_A;
constexpr uint32_t OFF_YL = OFF_YH + SZ_X;
constexpr uint32_t OFF_BAR = OFF_YL + SZ_X;
// barriers (8 bytes each): full[3], empty[3], inv_full, inv_empty, dfull, yready, xfull, xready
enum { B_FULL = 0, B_EMPTY = NSTAGE, B_INVF = 2 * NSTAGE, B_INVE, B_DFULL, B_YRDY, B_XFULL, B_XRDY, B_COUNT };
constexpr uint32_t OFF_MISC = OFF_BAR + 8 * B_COUNT;  // TMEM slot, abort word
constexpr uint32_t SMEM = OFF_MISC + 16;
static_assert(SZ_STAGE % 1024 == 0, "TMA destinations stay 1024-byte aligned");

constexpr uint32_t A_MN = 128, A_K = (NB2 / 8) * 128;  // A tiles: core matrices 128 B apart along MN
constexpr uint32_t X_N = 128, X_K = (NT / 8) * 128;    // X / Y tiles (MN-major)
constexpr uint32_t TM_D0 = 0, TM_D1 = NT, TM_X = 2 * NT, TM_COLS = 128;
constexpr size_t INV_SMEM = 2 * sizeof(float) * NB2 * (NB2 + 1);
constexpr uint32_t WAIT_LIMIT = 1u << 26;

// One launch serves up to MAXP problems (the layers of a batched natural
// gradient); a block finds its problem by binary search over the prefix of the
// blocks each problem takes.
struct PackBatch {
  const __nv_bfloat16* A[MAXP];
  int64_t ldA[MAXP], n[MAXP];
  uint8_t* tiles[MAXP];
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
  int vb[MAXP];
  int blk0[MAXP + 1];
  int np, trans;
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
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(bar), "r"(parity)
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
__global__ void __launch_bounds__(256) pack_tiles_kernel(const __grid_constant__ PackBatch pb) {
  extern __shared__ __align__(16) uint8_t img[];
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
__global__ void __launch_bounds__(NB2) diag_inverse_layout_kernel(const __grid_constant__ InvBatch ib) {
  extern __shared__ float dsm[];
  float (*U)[NB2 + 1] = reinterpret_cast<float (*)[NB2 + 1]>(dsm);
  float (*Xs)[NB2 + 1] = reinterpret_cast<float (*)[NB2 + 1]>(dsm + NB2 * (NB2 + 1));
  const int mat = find_problem(ib.blk0, ib.nm, (int)blockIdx.x);
  const __nv_bfloat16* A = ib.A[mat];
  const int64_t ldA_ = ib.ld[mat], n = ib.n[mat];
  const int b = (int)blockIdx.x - ib.blk0[mat], q = threadIdx.x;
  const int64_t b0 = (int64_t)b * NB2;
  const int nb = (int)mn<int64_t>(NB2, n - b0);
  for (int idx = q; idx < NB2 * NB2; idx += NB2) {
    const int r = idx / NB2, l = idx % NB2;
    float v = (r == l) ? 1.f : 0.f;
    if (r < nb && l < nb) v = (l >= r) ? __bfloat162float(A[(b0 + r) * ldA_ + b0 + l]) : 0.f;
    U[r][l] = v;
  }
  __syncthreads();
  // column q of U^-1 by back substitution; four partial sums break the FMA chain
  for (int r = NB2 - 1; r >= 0; --r) {
    float s0 = (r == q) ? 1.f : 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
    int l = r + 1;
    for (; l + 3 < NB2; l += 4) {
      s0 -= U[r][l] * Xs[l][q];
      s1 -= U[r][l + 1] * Xs[l + 1][q];
      s2 -= U[r][l + 2] * Xs[l + 2][q];
      s3 -= U[r][l + 3] * Xs[l + 3][q];
    }
    for (; l < NB2; ++l) s0 -= U[r][l] * Xs[l][q];
    Xs[r][q] = ((s0 + s1) + (s2 + s3)) / U[r][r];
  }
  __syncthreads();
  uint8_t* o = ib.inv[mat] + (size_t)b * 4 * SZ_A;
  for (int it = q; it < NB2 * (NB2 / 8); it += NB2) {
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

__global__ void __launch_bounds__(TPB, 1) trsm_persist_kernel(const __grid_constant__ SolveBatch sbt) {
  extern __shared__ __align__(1024) uint8_t sm[];
  const int prob = find_problem(sbt.blk0, sbt.np, (int)blockIdx.x);
  const int bx = (int)blockIdx.x - sbt.blk0[prob];  // this CTA's column group within its problem
  const uint8_t* tiles = sbt.tiles[prob];
  const int trans = sbt.trans;
  float* B = sbt.B[prob];
  const int64_t rs = sbt.rs[prob], cs = sbt.cs[prob], n = sbt.n[prob], N = sbt.N[prob];
  const __nv_bfloat16* inv = sbt.inv[prob];
  __nv_bfloat16* xws = sbt.xws[prob];
  int* err = sbt.err;
  const int vb = sbt.vb[prob];
  const uint32_t sb = tc::smem_u32(sm);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + OFF_MISC);
  volatile int* abort_ = reinterpret_cast<volatile int*>(sm + OFF_MISC + 4);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nblk = (int)cdiv(n, NB2);
  const int64_t c0 = (int64_t)bx * NT;
  const int nc = (int)mn<int64_t>(NT, N - c0);
  // this CTA's bf16 copies of its solved blocks: nblk tiles of 8 KB (MN-major B operand)
  uint8_t* xmine = reinterpret_cast<uint8_t*>(xws) + (size_t)bx * nblk * SZ_X;

  if (warp == 0) tc::tmem_alloc(tslot, TM_COLS);
  if (tid == 0) {
    for (int i = 0; i < NSTAGE; ++i) {
      tc::mbar_init(reinterpret_cast<uint64_t*>(sm + OFF_BAR) + B_FULL + i, 1);
      tc::mbar_init(reinterpret_cast<uint64_t*>(sm + OFF_BAR) + B_EMPTY + i, 1);
    }
    tc::mbar_init(reinterpret_cast<uint64_t*>(sm + OFF_BAR) + B_INVF, 1);
    tc::mbar_init(reinterpret_cast<uint64_t*>(sm + OFF_BAR) + B_INVE, 1);
    tc::mbar_init(reinterpret_cast<uint64_t*>(sm + OFF_BAR) + B_DFULL, 1);
    tc::mbar_init(reinterpret_cast<uint64_t*>(sm + OFF_BAR) + B_YRDY, 4);
    tc::mbar_init(reinterpret_cast<uint64_t*>(sm + OFF_BAR) + B_XFULL, 1);
    tc::mbar_init(reinterpret_cast<uint64_t*>(sm + OFF_BAR) + B_XRDY, 4);
    *abort_ = 0;
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tm = *tslot;

  if (warp == 4) {
    // ---------------- producer ----------------
    if (lane == 0) {
      uint32_t g = 0;
      bool ok = true;
      for (int row = 0; row < nblk && ok; ++row) {
        const int jb = trans ? row : nblk - 1 - row;
        for (int i = 0; i < row && ok; ++i) {
          // solved blocks, most recent last: forward s = 0.., backward s = nblk-1 ..
          const int s = trans ? i : nblk - 1 - i;
          if (i == row - 1) ok = wait_phase(bar_addr(sb, B_XRDY), (row - 1) & 1, abort_);
          const int st = (int)(g % NSTAGE);
          if (ok && g >= NSTAGE) ok = wait_phase(bar_addr(sb, B_EMPTY + st), ((g / NSTAGE) - 1) & 1, abort_);
          if (!ok) break;
          const uint32_t full = bar_addr(sb, B_FULL + st);
          const uint32_t dst = sb + (uint32_t)st * SZ_STAGE;
          arrive_expect(full, SZ_STAGE);
          // op(A)_{j,s} is the packed image of A block (min, max) of (j, s)
          const int ta = jb < s ? jb : s, tb = jb < s ? s : jb;
          bulk_load(dst, tiles + (size_t)(tb * (tb - 1) / 2 + ta) * SZ_A, SZ_A, full);
          bulk_load(dst + SZ_A, xmine + (size_t)s * SZ_X, SZ_X, full);
          ++g;
        }
        if (!ok) break;
        if (row > 0) ok = wait_phase(bar_addr(sb, B_INVE), (row - 1) & 1, abort_);
        if (!ok) break;
        const uint32_t invf = bar_addr(sb, B_INVF);
        arrive_expect(invf, 2 * SZ_A);
        const uint8_t* src = reinterpret_cast<const uint8_t*>(inv) + (size_t)jb * 4 * SZ_A + (trans ? 2 * SZ_A : 0);
        bulk_load(sb + OFF_IH, src, SZ_A, invf);
        bulk_load(sb + OFF_IL, src + SZ_A, SZ_A, invf);
      }
      // every copy issued was consumed by the MMA warp unless a wait gave up
      if (!ok) {
        for (uint32_t q = g > NSTAGE ? g - NSTAGE : 0; q < g; ++q)
          wait_phase(bar_addr(sb, B_FULL + (int)(q % NSTAGE)), (q / NSTAGE) & 1, abort_);
        if (err) atomicExch(err, IFK_ERR_TIMEOUT);
      }
    }
  } else if (warp == 5) {
    // ---------------- MMA issue ----------------
    if (lane == 0) {
      uint32_t g = 0;
      bool ok = true;
      const uint32_t idK = tc::idesc_bf16(128, NT, trans != 0, true);
      const uint32_t idI = tc::idesc_bf16(128, NT, trans != 0, true);
      for (int row = 0; row < nblk && ok; ++row) {
        const uint32_t dbuf = (row & 1) ? TM_D1 : TM_D0;
        for (int i = 0; i < row && ok; ++i) {
          const int st = (int)(g % NSTAGE);
          ok = wait_phase(bar_addr(sb, B_FULL + st), (g / NSTAGE) & 1, abort_);
          if (!ok) break;
          tc::fence_after();
          const uint32_t a0 = sb + (uint32_t)st * SZ_STAGE, x0 = a0 + SZ_A;
          const uint64_t ad = tc::sdesc(a0, A_K, A_MN), bd = tc::sdesc(x0, X_K, X_N);
          tc::mma_bf16(tm + dbuf, ad, bd, idK, i > 0 ? 1u : 0u);
#pragma unroll
          for (int k = 1; k < NB2 / 16; ++k)
            tc::mma_bf16(tm + dbuf, ad + tc::doff(k * 2 * A_K), bd + tc::doff(k * 2 * X_K), idK, 1u);
          commit_to(bar_addr(sb, B_EMPTY + st));
          ++g;
        }
        if (!ok) break;
        commit_to(bar_addr(sb, B_DFULL));
        ok = wait_phase(bar_addr(sb, B_YRDY), row & 1, abort_) && wait_phase(bar_addr(sb, B_INVF), row & 1, abort_);
        if (!ok) break;
        tc::fence_after();
        {
          const uint64_t ah = tc::sdesc(sb + OFF_IH, A_K, A_MN), al = tc::sdesc(sb + OFF_IL, A_K, A_MN);
          const uint64_t bh = tc::sdesc(sb + OFF_YH, X_K, X_N), bl = tc::sdesc(sb + OFF_YL, X_K, X_N);
#pragma unroll
          for (int k = 0; k < NB2 / 16; ++k) {
            const uint64_t da = tc::doff(k * 2 * A_K), dx = tc::doff(k * 2 * X_K);
            tc::mma_bf16(tm + TM_X, ah + da, bh + dx, idI, k > 0);
            tc::mma_bf16(tm + TM_X, ah + da, bl + dx, idI, 1);
            tc::mma_bf16(tm + TM_X, al + da, bh + dx, idI, 1);
          }
        }
        commit_to(bar_addr(sb, B_XFULL));
        commit_to(bar_addr(sb, B_INVE));
      }
      if (!ok && err) atomicExch(err, IFK_ERR_TIMEOUT);
    }
  } else {
    // ---------------- epilogue: warps 0-3, thread r = row of the block ----------------
    const int r = tid;
    const uint32_t lane_base = tm + ((uint32_t)(warp * 32) << 16);
    bool ok = true;
    for (int row = 0; row < nblk && ok; ++row) {
      const int jb = trans ? row : nblk - 1 - row;
      const int64_t j0 = (int64_t)jb * NB2;
      const int nj = (int)mn<int64_t>(NB2, n - j0);
      ok = wait_phase(bar_addr(sb, B_DFULL), row & 1, abort_);
      if (!ok) break;
      tc::fence_after();
      float d[32];
      if (row > 0) {
        tc::tmem_ld32(lane_base + ((row & 1) ? TM_D1 : TM_D0), d);
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) d[e] = 0.f;
      }
      float bv[NT];
      if (cs == 1 && vb) {
#pragma unroll
        for (int g = 0; g < NT / 4; ++g) {
          const float4 x = r < nj ? ld4(B + (j0 + r) * rs + c0 + 4 * g, nc - 4 * g) : make_float4(0.f, 0.f, 0.f, 0.f);
          bv[4 * g] = x.x; bv[4 * g + 1] = x.y; bv[4 * g + 2] = x.z; bv[4 * g + 3] = x.w;
        }
      } else {
#pragma unroll
        for (int c = 0; c < NT; ++c) bv[c] = (r < nj && c < nc) ? B[(j0 + r) * rs + (c0 + c) * cs] : 0.f;
      }
#pragma unroll
      for (int g = 0; g < NT / 8; ++g) {
        float hi[8], lo[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) tc::split_bf16(bv[g * 8 + e] - d[g * 8 + e], hi[e], lo[e]);
        const uint32_t off = tc::cm_off<false>(g * 8, r, X_N, X_K);
        st16(sb + OFF_YH + off, pack8(hi));
        st16(sb + OFF_YL + off, pack8(lo));
      }
      tc::fence_async_smem();
      tc::fence_before();
      __syncwarp();
      if (lane == 0) arrive(bar_addr(sb, B_YRDY));
      ok = wait_phase(bar_addr(sb, B_XFULL), row & 1, abort_);
      if (!ok) break;
      tc::fence_after();
      float x[32];
      tc::tmem_ld32(lane_base + TM_X, x);
      if (r < nj) {
        if (cs == 1 && vb) {
#pragma unroll
          for (int g = 0; g < NT / 4; ++g)
            st4(B + (j0 + r) * rs + c0 + 4 * g, make_float4(x[4 * g], x[4 * g + 1], x[4 * g + 2], x[4 * g + 3]),
                nc - 4 * g);
        } else {
#pragma unroll
          for (int c = 0; c < NT; ++c)
            if (c < nc) B[(j0 + r) * rs + (c0 + c) * cs] = x[c];
        }
      }
      // bf16 copy of X_j for the later block rows of this CTA (rows past n and
      // columns past N are exact zeros: their Y is zero)
      uint8_t* xo = xmine + (size_t)jb * SZ_X;
#pragma unroll
      for (int g = 0; g < NT / 8; ++g)
        *reinterpret_cast<uint4*>(xo + tc::cm_off<false>(g * 8, r, X_N, X_K)) = pack8(x + g * 8);
      asm volatile("fence.proxy.async.global;" ::: "memory");
      tc::fence_before();
      __syncwarp();
      if (lane == 0) arrive(bar_addr(sb, B_XRDY));
    }
    if (!ok && err) atomicExch(err, IFK_ERR_TIMEOUT);
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after();
    tc::tmem_free(tm, TM_COLS);
  }
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

size_t trsm_persist_inverse_bytes(int64_t n) { return (size_t)cdiv(n, NB2) * 4 * SZ_A; }

size_t trsm_persist_workspace(int64_t n, int64_t N) {
  const size_t nblk = (size_t)cdiv(n, NB2);
  return (size_t)cdiv(N, NT) * nblk * SZ_X + nblk * (nblk - 1) / 2 * SZ_A;
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
    diag_inverse_layout_kernel<<<(unsigned)acc, NB2, INV_SMEM, s>>>(ib);
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
  for (int base = 0; base < np; base += MAXP) {
    const int cnt = np - base < MAXP ? np - base : MAXP;
    PackBatch pb;
    SolveBatch sbt;
    pb.np = sbt.np = cnt;
    pb.trans = sbt.trans = trans;
    sbt.err = err;
    int tacc = 0, cacc = 0;
    for (int q = 0; q < cnt; ++q) {
      const TrsmProblem& P = p[base + q];
      const int64_t nblk = cdiv(P.n, NB2);
      // workspace of a problem: bf16 X copies | packed tiles
      uint8_t* w = (uint8_t*)P.ws;
      __nv_bfloat16* xws = (__nv_bfloat16*)w;
      w += (size_t)cdiv(P.N, NT) * nblk * SZ_X;
      pb.A[q] = P.A;
      pb.ldA[q] = P.ldA;
      pb.n[q] = P.n;
      pb.tiles[q] = w;
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
      // 16-byte vector access to rows of B needs 16-byte aligned rows
      sbt.vb[q] = (((uintptr_t)P.B % 16) == 0 && (P.rs * 4) % 16 == 0) ? 1 : 0;
      sbt.blk0[q] = cacc;
      cacc += (int)cdiv(P.N, NT);
    }
    pb.blk0[cnt] = tacc;
    sbt.blk0[cnt] = cacc;
    if (tacc > 0) {
      pack_tiles_kernel<<<(unsigned)tacc, 256, SZ_A, s>>>(pb);
      IFK_CUDA_TRY(cudaGetLastError());
    }
    if (cacc > 0) {
      trsm_persist_kernel<<<(unsigned)cacc, TPB, SMEM, s>>>(sbt);
      IFK_CUDA_TRY(cudaGetLastError());
    }
  }
  return IFK_OK;
}

int trsm_persist_run(const __nv_bfloat16* A, int64_t ldA, int trans, float* B, int64_t rs, int64_t cs, int64_t n,
                     int64_t N, const void* inv, void* ws, int* err, cudaStream_t s) {
  const TrsmProblem p{A, ldA, B, rs, cs, n, N, inv, ws};
  return trsm_persist_run_many(1, &p, trans, err, s);
}

}  // namespace ifk
