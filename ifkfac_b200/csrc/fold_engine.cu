// Persistent streaming-TSQR fold on the tensor cores (IFK_PREC_BF16 path).
//
// The fold R <- qr([R; X]).R is cut into tasks COL(f, t, cb): fold f, row
// sub-tile t (SUB = 256 rows) and column block cb (WB = 128 columns, i.e. two
// panels of NB = 64).  One CTA per SM takes tickets from a global counter in
// wave order (t + cbw * cb), which is a topological order of the dependencies:
//   COL(f, t, cb) applies panel k < 2cb of sub-tile t once that panel is
//   published by COL(f, t, k/2) and COL(f, t-1, cb) has applied its own panel
//   k (the R rows of panel k in block cb are then final for sub-tile t-1: a
//   progress counter per task), and factors each 16-column leaf of its own
//   panels as COL(f, t-1, cb) finishes the same rows of the R diagonal block.
//   Sub-tile t so trails sub-tile t-1 by one leaf.
// A task only waits for lower tickets, which were handed to CTAs already
// running, so the schedule cannot deadlock; every wait is bounded anyway and
// reports IFK_ERR_TIMEOUT.
//
// A task keeps its 256 x 128 block of X in TMEM as an fp32 master (D3) and a
// bf16 operand image of it in shared memory.  Applying panel k (compact WY:
// Y_k, T_k published as ready-to-copy shared-memory images) is
//   D1 = X^T Y (tcgen05, K = 256)  ->  W^T = D1 + R[k rows, cb]^T
//   D2 = W^T T (3-term bf16 split) ->  R[k rows, cb] -= D2^T
//   D3 += -Y W2 (accumulates into the fp32 master in TMEM)
// After the applies the task factors its own two panels (panel.cuh) from the
// fp32 master, publishes their Y / T images and R diagonal blocks, applies the
// first to the second half of the block, and marks itself done.  X is read
// from the caller's chunk once; there is no working copy in global memory.
#include <cstring>

#include "ifk_common.cuh"
#include "ifk_internal.h"
#include "panel.cuh"
#include "tc.cuh"

namespace ifk {

namespace {

constexpr int WB = 128;   // columns of a task
constexpr int TPB = 256;  // 8 warps; warps w and w + 4 share TMEM lanes 32(w%4)..+31
static_assert(TPB == panel::PT2, "the persistent fold runs the panel with all its threads");
constexpr int MAXW = 1536;  // waves per launch (the table of wave offsets in the launch parameters)
// Ticket order: wave d = t + cbw * cb (then by fold and t).  Any positive
// weights give a topological order of the dependencies.  The weight sets how
// far a column block's tasks trail the block to their left: a task handed out
// long before the panels it applies are published only waits, one handed out
// late delays the panel chain.  The next block's panels come about three
// sub-tile steps after a block's (the sub-tiles trail one another by a leaf,
// a block by two panels plus applies); measured on the config-2 fold (8.6 ms
// at weight 8 against 9.9 at 2, 9.3 at 3, 8.8 at 12 and 12.4 at 32), the weight
// is CBW_TARGET, lowered per launch where the wave table would overflow.
constexpr int CBW_TARGET = 8;
// Sub-tiles per launch piece (callers split longer folds): the limit that weight
// 2 and a 384-wave table gave, so workspaces keep their size.
constexpr int PIECE_WAVES = 384, PIECE_CBW = 2;

// The sub-tiles t of wave d for a fold of T sub-tiles and CB column blocks:
// t = tlo, tlo + cbw, ... (cnt of them), column block (d - t) / cbw.
__host__ __device__ __forceinline__ void wave_range(int d, int T, int CB, int cbw, int* tlo, int* cnt) {
  int lo = d - cbw * (CB - 1);
  if (lo < 0) lo = 0;
  lo += (d - lo) % cbw;
  const int hi = d < T - 1 ? d : T - 1;
  *tlo = lo;
  *cnt = hi >= lo ? (hi - lo) / cbw + 1 : 0;
}
__host__ __device__ __forceinline__ int num_waves(int T, int CB, int cbw) { return T + cbw * (CB - 1); }
using panel::LDP;
using panel::PanelSmem;

// published per (fold, sub-tile, panel): Y image (32 KB) + T hi / lo images (8 KB each)
constexpr uint32_t YIMG = SUB * NB * 2;
constexpr uint32_t TIMG = NB * NB * 2;
constexpr uint32_t PIMG = YIMG + 2 * TIMG;

// Shared memory: a union of the apply operands and the panel workspace, then
// image buffer 0.  The apply phase uses two image buffers (panel k's images in
// one while panel k + 1's arrive in the other by a bulk copy) and a staging
// area for the next panel's R rows; the panel phase builds its own images in
// buffer 0.
constexpr uint32_t SZ_A1 = WB * SUB * 2;     // X^T bf16, MN-major (mn = column c, k = row i)
constexpr uint32_t SZ_A2 = WB * NB * 2;      // W^T hi / lo, K-major (mn = c, k = j)
constexpr uint32_t OFF_A1 = 0;
constexpr uint32_t OFF_A2H = OFF_A1 + SZ_A1;
constexpr uint32_t OFF_A2L = OFF_A2H + SZ_A2;
constexpr uint32_t OFF_B3 = OFF_A2H;          // W2 bf16, K-major: over W^T hi once GEMM2 has completed
constexpr uint32_t OFF_IMG1 = OFF_A2L + SZ_A2;                 // image buffer 1 (apply phase)
constexpr uint32_t OFF_RN = OFF_IMG1 + PIMG;                   // next panel's R rows, fp32 [j][column]
constexpr uint32_t SZ_RN = NB * WB * 4;
constexpr uint32_t APPLY_END = OFF_RN + SZ_RN;
constexpr uint32_t UNION = ((sizeof(PanelSmem) > APPLY_END ? sizeof(PanelSmem) : APPLY_END) + 1023) / 1024 * 1024;
constexpr uint32_t OFF_IMG0 = UNION;          // image buffer 0: Y (B of GEMM1, MN-major; A of GEMM3, K-major),
constexpr uint32_t IMG_TH = YIMG;             //   then T hi / lo, K-major (mn = j, k = l)
constexpr uint32_t IMG_TL = YIMG + TIMG;
constexpr uint32_t OFF_BAR = OFF_IMG0 + PIMG;
constexpr uint32_t SMEM = OFF_BAR + 64;
static_assert(SMEM <= 227 * 1024, "shared memory of one CTA");
static_assert(OFF_IMG1 % 1024 == 0 && OFF_IMG0 % 1024 == 0 && PIMG % 16 == 0, "bulk copy alignment");

constexpr uint32_t A1_MN = 128, A1_K = (WB / 8) * 128;  // 128, 2048
constexpr uint32_t Y_I = 1024, Y_J = 128;
constexpr uint32_t A2_MN = 128, A2_K = (WB / 8) * 128;  // 128, 2048
constexpr uint32_t B2_MN = 128, B2_K = (NB / 8) * 128;  // 128, 1024
constexpr uint32_t TM_D1 = 0, TM_D2 = 64, TM_D3 = 128, TM_COLS = 512;

// Element kinds of a segment: fp32 / bf16 rows, the identity, or an NCHW image read
// through im2col (XK_CONV + 2 * geometry slot + (bf16 ? 1 : 0)).
enum { XK_F32 = 0, XK_BF16 = 1, XK_IDENT = 2, XK_CONV = 8 };

#ifdef IFK_TRACE
// Diagnostic build only: per-task timestamps (globaltimer, ns), 28 int64 per task.
constexpr int TRN = 28;
__device__ long long g_trace[(1 << 14) * TRN];
__device__ int g_trace_n;
__device__ __forceinline__ long long gtime() {
  long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
#define TR_DECL long long tr[TRN] = {};
#define TR_SET(i, v) tr[i] = (v)
#define TR_ADD(i, v) tr[i] += (v)
#define TR_NOW() gtime()
__device__ long long g_wait_ns[1024];
#define WT_BEGIN const long long wt0_ = gtime();
#define WT_END g_wait_ns[blockIdx.x & 1023] += gtime() - wt0_;
#define TR_WAIT() g_wait_ns[blockIdx.x & 1023]
// nanoseconds thread 0 of each CTA spent in the leaf hooks of the own panels, waits excluded
__device__ long long g_hook_ns[1024];
#define HK_BEGIN const long long hk0_ = threadIdx.x == 0 ? gtime() - TR_WAIT() : 0;
#define HK_END if (threadIdx.x == 0) g_hook_ns[blockIdx.x & 1023] += gtime() - TR_WAIT() - hk0_;
#define TR_HOOK() g_hook_ns[blockIdx.x & 1023]
#define TR_FLUSH()                                                     \
  if (threadIdx.x == 0) {                                              \
    const int slot = atomicAdd(&g_trace_n, 1);                         \
    if (slot < (1 << 14))                                              \
      for (int q_ = 0; q_ < TRN; ++q_) g_trace[slot * TRN + q_] = tr[q_]; \
  }
#else
#define TR_DECL
#define TR_SET(i, v)
#define TR_ADD(i, v)
#define TR_NOW() 0
#define TR_FLUSH()
#define WT_BEGIN
#define WT_END
#define TR_WAIT() 0
#define HK_BEGIN
#define HK_END
#define TR_HOOK() 0
#endif

#ifdef IFK_TRACE
// Diagnostic build only: time (ns) of the phases of the applies, summed over all
// applies by thread 0 of each CTA; slot 8 counts applies.
__device__ unsigned long long g_apply_phase[16];
#define AP_DECL long long ap_last = gtime();
#define AP_MARK(i)                                                      \
  do {                                                                  \
    if (threadIdx.x == 0) {                                             \
      const long long t_ = gtime();                                     \
      atomicAdd(&g_apply_phase[i], (unsigned long long)(t_ - ap_last)); \
      ap_last = t_;                                                     \
    }                                                                   \
  } while (0)
#else
#define AP_DECL
#define AP_MARK(i) do { } while (0)
#endif

// A segment of a fold's rows: sub-tiles t0 .. of the fold, row_off rows of the
// fold before it.
struct PSeg {
  const void* X;
  int64_t ldX;          // im2col segments: the first image row (X is an NCHW image)
  int64_t rows, row_off;
  const int64_t* ridx;  // row i of the segment is row ridx[i] of X (null: row i)
  int64_t src_rows;     // rows of X (bound for ridx)
  int64_t cols;         // columns read from X; column cols (when < n) is ones
  int t0;
  int xkind;
  int tri;      // row i of the segment is zero left of column i
  float ident;  // diagonal value when xkind == XK_IDENT
};

struct PFold {
  float* R;
  int64_t ldR;
  int64_t n, rows_R;
  int T, K, CB, nseg;
  int seg0;      // first of its nseg segments in PFBatch::seg
  int* prog;     // [T][CB]: k < K: panels < k applied to the block's R rows; K + s: own-panel stage s
  int* pflag;    // [T][K]
  uint8_t* img;  // [T][K][PIMG]
};

struct PFBatch {
  PFold f[PFOLD_MAX_FOLDS];
  PSeg seg[PFOLD_MAX_BATCH_SEGS];
  int nf;
  int cbw;  // ticket-order weight of the column block
  int nwaves;
  int ntasks;
  int* ctr;     // ticket counter
  int* abort_;  // set when a wait gave up: every CTA stops
  int* status;  // caller's status word (may be null)
  uint32_t wait_limit;  // polls of a cross-CTA wait before it gives up
  int withhold;         // test only: the first panel of fold 0 is never published
  ConvGeo conv[PFOLD_MAX_CONV];  // geometry of the im2col segments
  int wave_off[MAXW + 1];
};
static_assert(sizeof(PFBatch) <= 32000, "launch parameters of one persistent fold launch (limit 32764 bytes)");

__device__ __forceinline__ void st16(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void store8(uint32_t addr, const float (&v)[8]) {
  st16(addr, make_uint4(tc::pack_bf16(v[0], v[1]), tc::pack_bf16(v[2], v[3]), tc::pack_bf16(v[4], v[5]),
                        tc::pack_bf16(v[6], v[7])));
}

using tc::tmem_st32;
using tc::tmem_st_wait;

// Bulk copy of a panel's images from shared to global memory by the TMA engine
// (one thread; completion through the bulk-group counter).
__device__ __forceinline__ void bulk_store(void* gdst, uint32_t ssrc, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(ssrc), "r"(bytes)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait for this thread's bulk stores, then release *flag to other CTAs (the
// proxy fence orders the copy engine's writes before the release store).
// release == false (the test-only withheld panel) waits for the stores alone.
__device__ __forceinline__ void bulk_publish(int* flag, bool release = true) {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  asm volatile("fence.proxy.async.global;" ::: "memory");
  if (release) asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(flag), "r"(1) : "memory");
}

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release(int* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Thread 0 waits for *flag >= target (bounded); the CTA learns the outcome through smem.
__device__ __forceinline__ bool cta_wait_ge(const int* flag, int target, const PFBatch& b, int* s_ok) {
  if (threadIdx.x == 0) {
    WT_BEGIN
    int ok = 0;
    for (uint32_t it = 0; it < b.wait_limit; ++it) {
      if (ld_acquire(flag) >= target) {
        ok = 1;
        break;
      }
      if ((it & 31) == 31 && *((volatile int*)b.abort_)) break;
      __nanosleep(64);
    }
    if (!ok) {
      atomicExch(b.abort_, 1);
      if (b.status) atomicExch(b.status, IFK_ERR_TIMEOUT);
    }
    *s_ok = ok;
    WT_END
  }
  __syncthreads();
  const bool ok = *(volatile int*)s_ok != 0;
  __syncthreads();
  return ok;
}
__device__ __forceinline__ bool cta_wait_flag(const int* flag, const PFBatch& b, int* s_ok) {
  return cta_wait_ge(flag, 1, b, s_ok);
}

// Publish v at *flag once every thread's global writes so far are visible:
// the barrier orders them before thread 0's release store, and a gpu-scope
// release is cumulative over what happens before it (no separate fence).
__device__ __forceinline__ void cta_publish_value(int* flag, int v) {
  __syncthreads();
  if (threadIdx.x == 0) st_release(flag, v);
}

// Own-panel stages of a task in its progress counter (after the apply stages
// 0 .. K): panel q of the block publishes the R diagonal block rows of its leaf
// s at stage K + 1 + 5q + s as soon as that leaf ends; stage K + 5 marks the
// first panel applied to the block's second half and K + 9 the task done.
__host__ __device__ constexpr int stage_leaf(int K, int q, int s) { return K + 1 + 5 * q + s; }
__host__ __device__ constexpr int stage_half(int K) { return K + 5; }
__host__ __device__ constexpr int stage_done(int K) { return K + 9; }

// Leaf hooks of the fold's own panels: leaf s of sub-tile t starts once
// sub-tile t - 1 has published the R diagonal block rows of its leaf s (those
// rows are then final for t - 1), so consecutive sub-tiles factor the same
// panel one leaf apart; the rows go back to R when the leaf ends.  When a leaf
// ends and sub-tile t - 1 has already published the next leaf's rows, they are
// copied in at once (cp.async, zero-filled like the plain load), so the next
// leaf finds them without a wait or a load round trip.  Only leaf s touches
// rows 16s .. 16s + 15 of the block, so the early copy overwrites nothing in use.
struct FoldLeafHook {
  float* R;
  int64_t ldR, c0;
  int nbk, stage0;
  const int* prev_prog;  // null for the first sub-tile
  int* prog;
  const PFBatch* b;
  int* s_ok;
  int* s_pre;  // shared flag: the rows of the next leaf were copied in early
  bool published = false;  // this leaf's rows were stored and published by rows_final
  template <class SM>
  __device__ __forceinline__ void copy_rows(SM& S, int s) {
    const int L0 = s * panel::LEAF;
    for (int idx = threadIdx.x; idx < panel::LEAF * NB; idx += TPB) {
      const int i = L0 + idx / NB, j = idx % NB;
      const bool v = i < nbk && j < nbk && j >= i;
      const uint32_t dst = (uint32_t)__cvta_generic_to_shared(&S.Rk[i * LDP + j]);
      asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst),
                   "l"(v ? R + (c0 + i) * ldR + c0 + j : R), "r"(v ? 4 : 0)
                   : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  template <class SM>
  __device__ __forceinline__ bool before_leaf(SM& S, int s) {
    HK_BEGIN
    if (s > 0 && *(volatile int*)s_pre) {
      // copied in when leaf s - 1 ended, after sub-tile t - 1 had published them
      asm volatile("cp.async.wait_all;" ::: "memory");
      __syncthreads();
      HK_END
      return true;
    }
    if (prev_prog && !cta_wait_ge(prev_prog, stage0 + s, *b, s_ok)) return false;
    const int L0 = s * panel::LEAF;
    for (int idx = threadIdx.x; idx < panel::LEAF * NB; idx += TPB) {
      const int i = L0 + idx / NB, j = idx % NB;
      S.Rk[i * LDP + j] = (i < nbk && j < nbk && j >= i) ? R[(c0 + i) * ldR + c0 + j] : 0.f;
    }
    __syncthreads();
    HK_END
    return true;
  }
  template <class SM>
  __device__ __forceinline__ void store_rows(SM& S, int s) {
    const int L0 = s * panel::LEAF;
    for (int idx = threadIdx.x; idx < panel::LEAF * NB; idx += TPB) {
      const int i = L0 + idx / NB, j = idx % NB;
      if (i < nbk && j < nbk && j >= i) R[(c0 + i) * ldR + c0 + j] = S.Rk[i * LDP + j];
    }
  }
  // The leaf's rows are final before the update of the panel's trailing columns:
  // they are published then, so sub-tile t + 1 can start the same leaf meanwhile.
  template <class SM>
  __device__ __forceinline__ void rows_final(SM& S, int s) {
    HK_BEGIN
    store_rows(S, s);
    cta_publish_value(prog, stage0 + s);
    published = true;
    HK_END
  }
  template <class SM>
  __device__ __forceinline__ void after_leaf(SM& S, int s) {
    HK_BEGIN
    if (!published) store_rows(S, s);
    // is the next leaf's input already published?  (thread 0's acquire, passed on
    // to the other threads by the barrier below)
    const int s1 = s + 1;
    if (threadIdx.x == 0)
      *s_pre = (s1 * panel::LEAF < nbk && (!prev_prog || ld_acquire(prev_prog) >= stage0 + s1)) ? 1 : 0;
    if (published) {
      __syncthreads();
    } else {
      cta_publish_value(prog, stage0 + s);
    }
    published = false;
    if (*(volatile int*)s_pre) copy_rows(S, s1);
    HK_END
  }
};

// fp32 values of segment row gi, columns gj .. gj + 31 of the fold (gi < rows and
// the valid count already bounded by the fold's width).  Gathered rows come from
// row ridx[gi] of X; an index outside X gives a zero row and IFK_ERR_ARG.
// Columns past X's own (cols) read 1 (the bias column) then 0.
__device__ __forceinline__ void load_row32(const PSeg& F, int64_t gi, int64_t gj, int valid, float (&v)[32],
                                           int* status, const ConvGeo* conv) {
  if (F.xkind == XK_IDENT) {
#pragma unroll
    for (int e = 0; e < 32; ++e) v[e] = (e < valid && gi == gj + e) ? F.ident : 0.f;
    return;
  }
  // an im2col segment without row indices starts at image row ldX (its launch piece)
  int64_t si = F.xkind >= XK_CONV ? gi + F.ldX : gi;
  if (F.ridx) {
    si = F.ridx[gi];
    if (si < 0 || si >= F.src_rows) {
      if (status) atomicExch(status, IFK_ERR_ARG);
#pragma unroll
      for (int e = 0; e < 32; ++e) v[e] = 0.f;
      return;
    }
  }
  const int64_t vm64 = F.cols - gj;  // columns of this group held by X
  const int vm = vm64 < valid ? (vm64 > 0 ? (int)vm64 : 0) : valid;
  if (F.xkind >= XK_CONV) {
    // im2col row si of the NCHW image: gathered element by element (zero padding)
    const ConvGeo& g = conv[(F.xkind - XK_CONV) >> 1];
    const bool bf = ((F.xkind - XK_CONV) & 1) != 0;
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      float x = 0.f;
      if (e < vm) {
        const int64_t off = conv_offset(g, si, gj + e);
        if (off >= 0)
          x = bf ? __bfloat162float(((const __nv_bfloat16*)F.X)[off]) : ((const float*)F.X)[off];
      }
      v[e] = x;
    }
  } else if (F.xkind == XK_BF16) {
    const __nv_bfloat16* p = (const __nv_bfloat16*)F.X + si * F.ldX + gj;
    const bool vec = vm >= 32 && ((((uintptr_t)p) & 15) == 0);
    if (vec) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 u = reinterpret_cast<const uint4*>(p)[q];
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          v[q * 8 + 2 * e] = __uint_as_float(w[e] << 16);
          v[q * 8 + 2 * e + 1] = __uint_as_float(w[e] & 0xFFFF0000u);
        }
      }
    } else {
#pragma unroll
      for (int e = 0; e < 32; ++e) v[e] = e < vm ? __bfloat162float(p[e]) : 0.f;
    }
  } else {
    const float* p = (const float*)F.X + si * F.ldX + gj;
    const bool vec = ((((uintptr_t)p) & 15) == 0);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      float4 x;
      if (vec) {
        x = ld4(p + 4 * q, vm - 4 * q);
      } else {
        x.x = 4 * q < vm ? p[4 * q] : 0.f;
        x.y = 4 * q + 1 < vm ? p[4 * q + 1] : 0.f;
        x.z = 4 * q + 2 < vm ? p[4 * q + 2] : 0.f;
        x.w = 4 * q + 3 < vm ? p[4 * q + 3] : 0.f;
      }
      v[4 * q] = x.x;
      v[4 * q + 1] = x.y;
      v[4 * q + 2] = x.z;
      v[4 * q + 3] = x.w;
    }
  }
  const int64_t oc = F.cols - gj;  // the column of ones, when inside this group
  if (oc >= 0 && oc < valid) {
#pragma unroll
    for (int e = 0; e < 32; ++e) v[e] = (e == oc) ? 1.f : v[e];  // constant indices: v stays in registers
  }
}

struct Ctx {
  uint8_t* sm;
  uint32_t sb;
  uint32_t tm;
  uint64_t* bar;     // MMA completion
  uint64_t* ibar;    // [2] image buffer loads
  int* s_next;       // shared flag: the next panel's R rows may be staged
  int* s_ready;      // shared flag: the next panel is published and its R rows are final
  uint32_t phase;
  uint32_t ipar;     // bit b: parity of the next load phase of image buffer b
  int ipend;         // lookahead thread: bit b set while a load into buffer b is in flight
  bool ok;
};
// The thread that polls ahead and issues the image loads (warp 1), so that its
// flag loads run beside thread 0's MMA issue.
constexpr int LA = 32;
__device__ __forceinline__ uint32_t img_off(int b) { return b ? OFF_IMG1 : OFF_IMG0; }

__device__ __forceinline__ void mma_wait(Ctx& c) {
  c.ok = tc::mbar_wait(c.bar, c.phase) && c.ok;
  c.phase ^= 1;
  tc::fence_after();
}

__device__ __forceinline__ void sync_for_mma() {
  tc::fence_async_smem();
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
}

// bf16 operand image A1 (X^T) from the fp32 master in TMEM (all 128 columns, both halves)
__device__ void refresh_a1(Ctx& c) {
  const int tid = threadIdx.x, warp = tid >> 5;
  {
    const int h = tid >> 7;  // warps 0-3: rows 0..127, warps 4-7: rows 128..255
    const int r = tid;
    const uint32_t base = c.tm + ((uint32_t)((warp & 3) * 32) << 16) + TM_D3 + h * WB;
#pragma unroll 1
    for (int q = 0; q < WB / 64; ++q) {
      float v[64];
      tc::tmem_ld64(base + q * 64, v);
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        float e8[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) e8[e] = v[g * 8 + e];
        store8(c.sb + OFF_A1 + tc::cm_off<false>(q * 64 + g * 8, r, A1_MN, A1_K), e8);
      }
    }
  }
}

// Thread 0: start the bulk copy of a published panel's images (Y, T hi, T lo,
// contiguous as in global memory) into image buffer b.  The panel's flag was
// acquired by this thread; the proxy fence orders that acquire before the
// copy engine's reads.
__device__ __forceinline__ void img_issue(Ctx& c, int b, const uint8_t* src) {
  asm volatile("fence.proxy.async.global;" ::: "memory");
  tc::mbar_expect_tx(c.ibar + b, PIMG);
  tc::bulk_g2s(c.sb + img_off(b), src, PIMG, c.ibar + b);
  c.ipend |= 1 << b;
}
// All threads: wait (bounded) for the load into image buffer b.
__device__ __forceinline__ void img_wait(Ctx& c, int b) {
  c.ok = tc::mbar_wait(c.ibar + b, (c.ipar >> b) & 1u) && c.ok;
  c.ipar ^= 1u << b;
  c.ipend &= ~(1 << b);
}

// Where apply_panel takes its images and R rows, and its lookahead to the next panel.
struct ApplyOpts {
  int buf = 0;                      // image buffer holding the panel's Y / T images
  bool rpre = false;                // the panel's R rows were staged in OFF_RN during the previous apply
  // Lookahead to the next panel (none when next_flag is null), checked by
  // thread 0 while GEMM1 runs: its images are loaded into the other buffer if
  // it is published, and its R rows (k0_next, nbk_next) are staged while
  // GEMM2 runs if prev_prog shows them final (prev_prog null: always final).
  const int* next_flag = nullptr;
  const uint8_t* next_img = nullptr;
  const int* prev_prog = nullptr;
  int prev_need = 0;
  int64_t k0_next = 0;
  int nbk_next = 0;
};

// Stage R rows k0 .. k0 + nbk - 1 of the block in OFF_RN (element (j, col) at
// j * WB + col) by asynchronous copies; entries outside the panel or the block
// are zero-filled.  With 16-byte aligned rows every thread copies 8 chunks of 4
// columns, else 32 single entries.  Each thread waits for its own copies
// (cp.async.wait_all) before a CTA barrier that precedes the reads.
__device__ __forceinline__ void stage_r_rows(const Ctx& c, const PFold& F, int64_t k0, int nbk, int64_t cs,
                                             int wc, int col, int jh) {
  if ((F.ldR & 3) == 0 && (((uintptr_t)F.R) & 15) == 0) {
#pragma unroll
    for (int m = 0; m < (NB * WB / 4) / TPB; ++m) {
      const int idx = (int)threadIdx.x + m * TPB;
      const int j = idx / (WB / 4), c4 = (idx % (WB / 4)) * 4;
      const int nv = j < nbk ? (wc - c4 < 4 ? (wc - c4 > 0 ? wc - c4 : 0) : 4) : 0;
      const uint32_t dst = c.sb + OFF_RN + (uint32_t)(j * WB + c4) * 4u;
      const float* src = nv ? F.R + (k0 + j) * F.ldR + cs + c4 : F.R;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(nv * 4) : "memory");
    }
  } else {
    const uint32_t dst = c.sb + OFF_RN + (uint32_t)((jh * 32) * WB + col) * 4u;
    const float* src = F.R + (k0 + jh * 32) * F.ldR + cs + col;
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      const bool v = jh * 32 + e < nbk && col < wc;
      asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst + (uint32_t)(e * WB * 4)),
                   "l"(v ? src + (int64_t)e * F.ldR : F.R), "r"(v ? 4 : 0)
                   : "memory");
    }
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

// Apply panel k (Y / T images in image buffer o.buf, A1 current) to the task's
// block; when skip_half0 the first 64 columns are the panel itself and are left
// alone in R.
__device__ __forceinline__ void apply_panel(Ctx& c, const PFold& F, int64_t k0, int nbk, int64_t cs, int wc,
                                            bool skip_half0, const ApplyOpts& o) {
  const int tid = threadIdx.x, warp = tid >> 5;
  const int col = tid & 127;   // trailing column of this thread == TMEM lane
  const int jh = tid >> 7;     // which 32 of the 64 panel columns this thread handles
  const uint32_t lane_base = c.tm + ((uint32_t)((warp & 3) * 32) << 16);
  const uint32_t img = c.sb + img_off(o.buf);
  AP_DECL
  if (tid == 0) {
    constexpr uint32_t id1 = tc::idesc_bf16(128, NB, true, true);
    const uint64_t ad = tc::sdesc(c.sb + OFF_A1, A1_K, A1_MN);
    const uint64_t bd = tc::sdesc(img, Y_I, Y_J);
#pragma unroll
    for (int s = 0; s < SUB / 16; ++s)
      tc::mma_bf16(c.tm + TM_D1, ad + tc::doff(s * 2 * A1_K), bd + tc::doff(s * 2 * Y_I), id1, s > 0);
    tc::commit(c.bar);
    AP_MARK(10);
  } else if (tid == LA) {
    // Lookahead: the next panel's images go into the other buffer if it is
    // published; its R rows are staged during GEMM2 if sub-tile t - 1 has
    // finished them.  When both hold, the next apply skips its flag waits.
    if (o.next_flag) {
      const bool pub = ld_acquire(o.next_flag) >= 1;
      if (pub) img_issue(c, o.buf ^ 1, o.next_img);
      const bool fin = !o.prev_prog || ld_acquire(o.prev_prog) >= o.prev_need;
      *c.s_next = fin;
      *c.s_ready = pub && fin;
    } else {
      *c.s_next = 0;
      *c.s_ready = 0;
    }
  }
  // this thread's 32 R entries, read once while GEMM1 runs (staged by the CTA
  // during the previous apply, or from global memory)
  const bool rcol = col < wc && !(skip_half0 && col < NB);
  float rr[32];
  if (o.rpre) {
    asm volatile("cp.async.wait_all;" ::: "memory");
    const float* rs = reinterpret_cast<const float*>(c.sm + OFF_RN) + (jh * 32) * WB + col;
#pragma unroll
    for (int e = 0; e < 32; ++e) rr[e] = rs[e * WB];
  } else {
    const float* rp = F.R + (k0 + jh * 32) * F.ldR + cs + col;
#pragma unroll
    for (int e = 0; e < 32; ++e) rr[e] = (jh * 32 + e < nbk && col < wc) ? rp[(int64_t)e * F.ldR] : 0.f;
  }
  mma_wait(c);
  AP_MARK(11);
  AP_MARK(1);
  {
    float w[32];
    tc::tmem_ld32(lane_base + TM_D1 + jh * 32, w);
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      float hi[8], lo[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) tc::split_bf16(w[g * 8 + e] + rr[g * 8 + e], hi[e], lo[e]);
      const uint32_t off = tc::cm_off<true>(col, jh * 32 + g * 8, A2_MN, A2_K);
      store8(c.sb + OFF_A2H + off, hi);
      store8(c.sb + OFF_A2L + off, lo);
    }
  }
  sync_for_mma();
  AP_MARK(2);
  if (tid == 0) {
    constexpr uint32_t id2 = tc::idesc_bf16(128, NB, false, false);
    const uint64_t ah = tc::sdesc(c.sb + OFF_A2H, A2_K, A2_MN);
    const uint64_t al = tc::sdesc(c.sb + OFF_A2L, A2_K, A2_MN);
    const uint64_t bh = tc::sdesc(img + IMG_TH, B2_K, B2_MN);
    const uint64_t bl = tc::sdesc(img + IMG_TL, B2_K, B2_MN);
#pragma unroll
    for (int s = 0; s < NB / 16; ++s) {
      const uint64_t da = tc::doff(s * 2 * A2_K), db = tc::doff(s * 2 * B2_K);
      tc::mma_bf16(c.tm + TM_D2, ah + da, bh + db, id2, s > 0);
      tc::mma_bf16(c.tm + TM_D2, ah + da, bl + db, id2, 1);
      tc::mma_bf16(c.tm + TM_D2, al + da, bh + db, id2, 1);
    }
    tc::commit(c.bar);
    AP_MARK(12);
  }
  // rr[] is in registers: the staging area takes the next panel's rows while GEMM2 runs
  if (*(volatile int*)c.s_next) stage_r_rows(c, F, o.k0_next, o.nbk_next, cs, wc, col, jh);
  AP_MARK(13);
  mma_wait(c);
  AP_MARK(3);
  float w[32];
  tc::tmem_ld32(lane_base + TM_D2 + jh * 32, w);
  // GEMM2 has completed: W2 goes over W^T hi
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = w[g * 8 + e];
    store8(c.sb + OFF_B3 + tc::cm_off<true>(col, jh * 32 + g * 8, A2_MN, A2_K), v);
  }
  // The new R rows go to global memory by 16-byte stores of whole row pieces when
  // R's rows are 16-byte aligned: this thread's column is transposed through the
  // A1 area, which GEMM3 does not read (GEMM1 has completed; the next refresh
  // rewrites it after a barrier).
  const bool vec_r = (F.ldR & 3) == 0 && (((uintptr_t)F.R) & 15) == 0;
  float* stg = reinterpret_cast<float*>(c.sm + OFF_A1);  // element (j, column) at j * WB + column
  if (vec_r) {
#pragma unroll
    for (int j = 0; j < 32; ++j) stg[(jh * 32 + j) * WB + col] = rr[j] - w[j];
  }
  sync_for_mma();
  AP_MARK(4);
  if (tid == 0) {
    // D3 += (-Y) W2: negate-A bit of the instruction descriptor
    constexpr uint32_t id3 = tc::idesc_bf16(128, WB, false, false) | (1u << 13);
    const uint64_t ad = tc::sdesc(img, Y_J, Y_I);
    const uint64_t bd = tc::sdesc(c.sb + OFF_B3, A2_K, A2_MN);
#pragma unroll
    for (int mh = 0; mh < 2; ++mh) {
#pragma unroll
      for (int s = 0; s < NB / 16; ++s)
        tc::mma_bf16(c.tm + TM_D3 + mh * WB, ad + tc::doff(mh * 16 * Y_I + s * 2 * Y_J),
                     bd + tc::doff(s * 2 * A2_K), id3, 1);
    }
    tc::commit(c.bar);
    AP_MARK(14);
  }
  // the block's R rows of the panel, written while GEMM3 runs; published by the
  // release that follows the next CTA barrier
  if (vec_r) {
    const int lo = skip_half0 ? NB : 0;  // first column written (NB is a multiple of 4)
#pragma unroll
    for (int m = 0; m < (NB * WB / 4) / TPB; ++m) {
      const int idx = tid + m * TPB;
      const int j = idx / (WB / 4), c4 = (idx % (WB / 4)) * 4;
      if (j < nbk && c4 >= lo && c4 < wc) {
        const float4 v = *reinterpret_cast<const float4*>(stg + j * WB + c4);
        float* dst = F.R + (k0 + j) * F.ldR + cs + c4;
        if (c4 + 4 <= wc) {
          *reinterpret_cast<float4*>(dst) = v;
        } else {  // the block's last columns
          dst[0] = v.x;
          if (c4 + 1 < wc) dst[1] = v.y;
          if (c4 + 2 < wc) dst[2] = v.z;
        }
      }
    }
  } else {
    float* rp = F.R + (k0 + jh * 32) * F.ldR + cs + col;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (jh * 32 + j < nbk && rcol) rp[(int64_t)j * F.ldR] = rr[j] - w[j];
  }
  mma_wait(c);
  AP_MARK(5);
}

__device__ void run_task(Ctx& c, const PFBatch& b, int f, int t, int cb, int* s_ok) {
  const PFold& F = b.f[f];
  TR_DECL
  TR_SET(0, f);
  TR_SET(1, t);
  TR_SET(2, cb);
  TR_SET(3, TR_NOW());
  TR_SET(20, TR_WAIT());
  TR_SET(24, TR_HOOK());
  const int tid = threadIdx.x, warp = tid >> 5;
  int si = 0;  // segment of sub-tile t
  const PSeg* SG = b.seg + F.seg0;
  while (si + 1 < F.nseg && SG[si + 1].t0 <= t) ++si;
  const PSeg& G = SG[si];
  const int64_t row0 = (int64_t)(t - G.t0) * SUB;  // first row of the sub-tile within its segment
  const int h = (int)mn<int64_t>(SUB, G.rows - row0);
  const int64_t cs = (int64_t)cb * WB;
  const int wc = (int)mn<int64_t>(WB, F.n - cs);
  // Rank bound: the rows folded so far, this sub-tile's included.  Past it the
  // sub-tile holds rounding residuals only, as long as every reflector consumed a
  // row of it.  A dependent column (duplicated, constant or all-zero activations)
  // has a zero or rounding-noise pivot, spends its reflector on that and leaves one
  // row direction of the sub-tile past the bound, which is dropped.  Once R is
  // square the loss is a few times this fold's bf16 rounding (measured, relative
  // in R^T R: 1.6e-3 with 5 of 3072 columns dependent, 3.7e-3 with 150, 5.9e-3
  // with 150 of 768; 1.1e-3 with every column factored).  The fp32 wave fold
  // factors every column and stays exact.
  const int64_t lim = mn<int64_t>(F.n, F.rows_R + G.row_off + row0 + h);
  const int kfirst = G.tri ? (int)(row0 / NB) : 0;
  int* prog = F.prog + (size_t)t * F.CB + cb;
  const int* prev_prog = t > 0 ? F.prog + (size_t)(t - 1) * F.CB + cb : nullptr;

  if (G.tri && cs + WB <= row0) {  // block entirely left of the sub-tile's diagonal: nothing to do
    cta_publish_value(prog, stage_done(F.K));
    return;
  }
  TR_SET(4, TR_NOW());

  // ---- X block -> fp32 master in TMEM (D3) + bf16 image A1 ----
  tc::fence_after();
  {
    const int hh = tid >> 7;
    const int r = tid;
    const uint32_t base = c.tm + ((uint32_t)((warp & 3) * 32) << 16) + TM_D3 + hh * WB;
#pragma unroll 1
    for (int q = 0; q < WB / 32; ++q) {
      float v[32];
      if (r < h) {
        load_row32(G, row0 + r, cs + q * 32, wc - q * 32, v, b.status, b.conv);
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] = 0.f;
      }
      tmem_st32(base + q * 32, v);
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        float e8[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) e8[e] = v[g * 8 + e];
        store8(c.sb + OFF_A1 + tc::cm_off<false>(q * 32 + g * 8, r, A1_MN, A1_K), e8);
      }
    }
  }
  tmem_st_wait();
  bool a1_valid = true;
  TR_SET(5, TR_NOW());

  // ---- apply the panels of sub-tile t left of this block ----
  // Panel k's images are in image buffer buf: loaded by a bulk copy started
  // during the previous apply when panel k was already published, else now.
  // The R rows of panel k + 1 are staged during apply k when sub-tile t - 1
  // has finished them by then.
  const int kend = (int)mn<int64_t>(2 * cb, cdiv(lim, NB));
  int buf = 0;
  bool rpre = false, ready = false;
#pragma unroll 1
  for (int k = kfirst; k < kend; ++k) {
#ifdef IFK_TRACE
    const long long w0 = TR_NOW();
#endif
    AP_DECL
    // the operand image of X depends on the previous apply only: refresh it before waiting
    if (!a1_valid) {
      // this thread's staged R rows are complete before the barrier (other threads read them)
      if (rpre) asm volatile("cp.async.wait_all;" ::: "memory");
      tc::fence_before();
      __syncthreads();
      tc::fence_after();
      // Panel k - 1 is applied to the block's R rows (written before the
      // barrier above): thread 0's release store publishes them before the
      // refresh, so sub-tile t + 1 can take them meanwhile.
      if (tid == 0) st_release(prog, k);
      refresh_a1(c);
      a1_valid = true;
    }
    AP_MARK(6);
    // skipped when the previous apply's lookahead saw panel k published and its R rows final
    if (!ready) {
      if (!cta_wait_flag(F.pflag + (size_t)t * F.K + k, b, s_ok)) return;
      AP_MARK(7);
      if (t > 0 && !cta_wait_ge(prev_prog, k + 1, b, s_ok)) return;
    }
    AP_MARK(9);
    TR_ADD(9, TR_NOW() - w0);
    TR_ADD(10, 1);
    if (tid == LA && !(c.ipend & (1 << buf))) {
      // not prefetched: this thread acquires the flag itself before the copy
      ld_acquire(F.pflag + (size_t)t * F.K + k);
      img_issue(c, buf, F.img + ((size_t)t * F.K + k) * PIMG);
    }
    img_wait(c, buf);
    sync_for_mma();
    if (!c.ok) return;
    AP_MARK(0);
    ApplyOpts o;
    o.buf = buf;
    o.rpre = rpre;
    if (k + 1 < kend) {
      o.next_flag = F.pflag + (size_t)t * F.K + k + 1;
      o.next_img = F.img + ((size_t)t * F.K + k + 1) * PIMG;
      o.prev_prog = prev_prog;
      o.prev_need = k + 2;
      o.k0_next = (int64_t)(k + 1) * NB;
      o.nbk_next = (int)mn<int64_t>(NB, F.n - (int64_t)(k + 1) * NB);
    }
    apply_panel(c, F, (int64_t)k * NB, (int)mn<int64_t>(NB, F.n - (int64_t)k * NB), cs, wc, false, o);
    rpre = *(volatile int*)c.s_next != 0;
    ready = *(volatile int*)c.s_ready != 0;
    buf ^= 1;
    a1_valid = false;
#ifdef IFK_TRACE
    if (tid == 0) atomicAdd(&g_apply_phase[8], 1ull);
#endif
  }
  // panels this sub-tile does not reach leave their R rows as they are
  cta_publish_value(prog, F.K);

  // ---- factor the block's own panels ----
  // Stages of this phase, published in prog and awaited from COL(t-1, cb):
  //   stage_leaf(K, q, s): rows of leaf s of panel 2cb + q's R diagonal block
  //   written; stage_half(K): panel 2cb applied to the block's second half (R
  //   rows of panel 2cb final); stage_done(K).  A panel this sub-tile skips
  //   (beyond its rank bound, or left of its diagonal in a trapezoidal fold) is
  //   skipped by every earlier sub-tile too, or by every later one, so its stages
  //   pass at once.
  TR_SET(6, TR_NOW());
  TR_SET(21, TR_WAIT());
  PanelSmem& S = *reinterpret_cast<PanelSmem*>(c.sm);
  int* pending_img = nullptr;  // flag of panel images whose bulk store is in flight
  // test only (IFK_FOLD_DEBUG_WITHHOLD): panel 0 of fold 0's first sub-tile is never
  // published, so every wait on it runs out and the launch reports IFK_ERR_TIMEOUT
  const bool withheld0 = b.withhold && f == 0 && t == 0 && cb == 0;
#pragma unroll 1
  for (int q = 0; q < 2; ++q) {
    const int kk = 2 * cb + q;
    const int64_t c0 = (int64_t)kk * NB;
    if (kk >= F.K || c0 >= lim || kk < kfirst) {
      cta_publish_value(prog, q == 0 ? stage_half(F.K) : stage_done(F.K));
      continue;
    }
    const int nbk = (int)mn<int64_t>(NB, F.n - c0);
    const int nact = (int)mn<int64_t>(nbk, lim - c0);
#ifdef IFK_TRACE
    const long long l0 = TR_NOW();
    TR_SET(18 + q, l0);
#endif
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    // panel columns from the fp32 master (rows beyond the sub-tile are zero there)
    {
      const int hh = tid >> 7;
      const int r = tid;
      const uint32_t base = c.tm + ((uint32_t)((warp & 3) * 32) << 16) + TM_D3 + hh * WB + q * NB;
      float v[NB];
      tc::tmem_ld64(base, v);
#pragma unroll
      for (int e = 0; e < NB; ++e) S.P[e * panel::SP + r] = v[e];
    }
    __syncthreads();
#ifdef IFK_TRACE
    const long long p0 = TR_NOW();
    const long long k0 = clock64();
    TR_ADD(8, p0 - l0);
#endif
    // the R diagonal block is read and written leaf by leaf (FoldLeafHook)
    FoldLeafHook hook{F.R, F.ldR, c0, nbk, stage_leaf(F.K, q, 0), t > 0 ? prev_prog : nullptr, prog, &b, s_ok,
                      c.s_ready};
    if (!panel::panel_factor<SUB>(S, nbk, nact, hook)) return;
#ifdef IFK_TRACE
    const long long p1 = TR_NOW();
    TR_ADD(11, p1 - p0);
    TR_ADD(26 + q, p1 - p0);
    TR_ADD(15, clock64() - k0);
#endif
    TR_ADD(12, 1);
    if (pending_img) {  // the first panel's bulk store must be done before its images are overwritten
      if (tid == 0) bulk_publish(pending_img, !withheld0);
      pending_img = nullptr;
      __syncthreads();
    }
    // Y image (bf16, K-major for GEMM3 / MN-major for GEMM1) and T hi / lo images;
    // lanes take consecutive rows, so the column reads of P are conflict-free
    for (int it = tid; it < SUB * (NB / 8); it += TPB) {
      const int i = it % SUB, j8 = it / SUB;
      float e8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) e8[e] = S.P[(j8 * 8 + e) * panel::SP + i];
      store8(c.sb + OFF_IMG0 + tc::cm_off<true>(i, j8 * 8, Y_I, Y_J), e8);
    }
    for (int it = tid; it < NB * (NB / 8); it += TPB) {
      const int j = it >> 3, l8 = it & 7;
      float hi[8], lo[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) tc::split_bf16(S.Tm[(l8 * 8 + e) * LDP + j], hi[e], lo[e]);
      const uint32_t off = tc::cm_off<true>(j, l8 * 8, B2_MN, B2_K);
      store8(c.sb + OFF_IMG0 + IMG_TH + off, hi);
      store8(c.sb + OFF_IMG0 + IMG_TL + off, lo);
    }
    // The images go by a bulk store.  The first panel's images are released only
    // before the second panel's overwrite them (the copy runs under the apply to
    // the block's second half and the second panel); the second panel's at once.
    tc::fence_async_smem();
    __syncthreads();
    if (tid == 0) bulk_store(F.img + ((size_t)t * F.K + kk) * PIMG, c.sb + OFF_IMG0, PIMG);
    const bool half = q == 0 && wc > NB;
    if (half) {
      TR_SET(16, TR_NOW());
      pending_img = F.pflag + (size_t)t * F.K + kk;
    } else {
      __syncthreads();
      if (tid == 0) bulk_publish(F.pflag + (size_t)t * F.K + kk, !(withheld0 && q == 0));
    }
    TR_ADD(13, TR_NOW() - p1);
    if (q == 0) {
#ifdef IFK_TRACE
      const long long h0 = TR_NOW();
#endif
      if (half) {
        // the first panel also acts on the block's second half
        if (t > 0 && !cta_wait_ge(prev_prog, stage_half(F.K), b, s_ok)) return;
        refresh_a1(c);
        sync_for_mma();
        apply_panel(c, F, c0, nbk, cs, wc, true, ApplyOpts{});  // own images: buffer 0
      }
      cta_publish_value(prog, stage_half(F.K));
      TR_SET(17, TR_NOW());
      TR_ADD(14, TR_NOW() - h0);
    }
  }
  if (pending_img) {
    if (tid == 0) bulk_publish(pending_img, !withheld0);
    __syncthreads();
  }
  tc::fence_before();
  cta_publish_value(prog, stage_done(F.K));
  TR_SET(7, TR_NOW());
  TR_SET(22, TR_WAIT());
  TR_SET(25, TR_HOOK());
  TR_FLUSH();
}

__device__ __forceinline__ void decode(const PFBatch& b, int tk, int* f, int* t, int* cb) {
  int lo = 0, hi = b.nwaves;  // wave_off[lo] <= tk < wave_off[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (b.wave_off[mid] <= tk) lo = mid;
    else hi = mid;
  }
  const int d = lo;
  int r = tk - b.wave_off[d];
  for (int q = 0; q < b.nf; ++q) {
    const PFold& F = b.f[q];
    int tlo, cnt;
    wave_range(d, F.T, F.CB, b.cbw, &tlo, &cnt);
    if (r < cnt) {
      *f = q;
      *t = tlo + r * b.cbw;
      *cb = (d - *t) / b.cbw;
      return;
    }
    r -= cnt;
  }
  *f = -1;
}

__global__ void __launch_bounds__(TPB, 1) fold_persistent_kernel(const __grid_constant__ PFBatch b) {
  extern __shared__ __align__(1024) uint8_t sm[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + OFF_BAR + 8);
  int* s_tk = reinterpret_cast<int*>(sm + OFF_BAR + 16);
  int* s_ok = reinterpret_cast<int*>(sm + OFF_BAR + 20);
  uint64_t* ibar = reinterpret_cast<uint64_t*>(sm + OFF_BAR + 24);  // [2]
  int* s_next = reinterpret_cast<int*>(sm + OFF_BAR + 40);
  int* s_ready = reinterpret_cast<int*>(sm + OFF_BAR + 44);
  const int tid = threadIdx.x, warp = tid >> 5;
  if (warp == 0) tc::tmem_alloc(tslot, TM_COLS);
  if (tid == 0) {
    tc::mbar_init(bar, 1);
    tc::mbar_init(ibar, 1);
    tc::mbar_init(ibar + 1, 1);
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  Ctx c;
  c.sm = sm;
  c.sb = tc::smem_u32(sm);
  c.tm = *tslot;
  c.bar = bar;
  c.ibar = ibar;
  c.s_next = s_next;
  c.s_ready = s_ready;
  c.phase = 0;
  c.ipar = 0;
  c.ipend = 0;
  c.ok = true;
#pragma unroll 1
  for (;;) {
    if (tid == 0) *s_tk = *((volatile int*)b.abort_) ? b.ntasks : atomicAdd(b.ctr, 1);
    __syncthreads();
    const int tk = *s_tk;
    __syncthreads();
    if (tk >= b.ntasks) break;
    int f, t, cb;
    decode(b, tk, &f, &t, &cb);
    if (f < 0) break;
    run_task(c, b, f, t, cb, s_ok);
    if (!c.ok) {
      if (tid == 0) {
        atomicExch(b.abort_, 1);
        if (b.status) atomicExch(b.status, IFK_ERR_TIMEOUT);
      }
      break;
    }
  }
  // a task that gave up may leave a bulk store of panel images, a bulk load of
  // images or staged R rows in flight: wait for them (bounded) before exiting
  if (tid == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  if (tid == LA) {
    for (int q = 0; q < 2; ++q)
      if (c.ipend & (1 << q)) tc::mbar_wait(ibar + q, (c.ipar >> q) & 1u);
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  tc::fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after();
    tc::tmem_free(c.tm, TM_COLS);
  }
}

int num_sms() {
  static thread_local int dev_cached = -1, sms = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (dev != dev_cached) {
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    if (cudaFuncSetAttribute(fold_persistent_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)SMEM) != cudaSuccess)
      return 0;
    dev_cached = dev;
  }
  return sms;
}

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

}  // namespace

#ifdef IFK_TRACE
extern "C" __attribute__((visibility("default"))) int ifk_trace_read(long long* dst, int max_tasks) {
  int n = 0;
  if (cudaMemcpyFromSymbol(&n, g_trace_n, sizeof(int)) != cudaSuccess) return -1;
  n = n < max_tasks ? n : max_tasks;
  if (n > (1 << 14)) n = 1 << 14;
  if (cudaMemcpyFromSymbol(dst, g_trace, (size_t)n * TRN * sizeof(long long)) != cudaSuccess) return -1;
  const int zero = 0;
  cudaMemcpyToSymbol(g_trace_n, &zero, sizeof(int));
  return n;
}
extern "C" __attribute__((visibility("default"))) int ifk_trace_apply_phases(unsigned long long* dst) {
  if (cudaMemcpyFromSymbol(dst, g_apply_phase, 16 * sizeof(unsigned long long)) != cudaSuccess) return -1;
  unsigned long long z[16] = {};
  cudaMemcpyToSymbol(g_apply_phase, z, sizeof(z));
  return 0;
}
extern "C" __attribute__((visibility("default"))) int ifk_trace_panel_phases(unsigned long long* dst) {
  if (cudaMemcpyFromSymbol(dst, panel::g_panel_phase, 16 * sizeof(unsigned long long)) != cudaSuccess) return -1;
  unsigned long long z[16] = {};
  cudaMemcpyToSymbol(panel::g_panel_phase, z, sizeof(z));
  return 0;
}
#endif

int64_t pfold_subtiles(const PFoldDesc& d) {
  int64_t t = 0;
  for (int s = 0; s < d.nseg; ++s) t += cdiv(d.seg[s].rows, SUB);
  return t;
}

int64_t pfold_max_subtiles(int64_t n) { return (int64_t)PIECE_WAVES - PIECE_CBW * (cdiv(n, WB) - 1); }

size_t pfold_workspace(int nf, const int64_t* subtiles, const int64_t* n) {
  size_t b = 256;
  for (int f = 0; f < nf; ++f) {
    if (subtiles[f] <= 0) continue;
    const int64_t T = subtiles[f], K = cdiv(n[f], NB), CB = cdiv(n[f], WB);
    b += align256((size_t)T * CB * 4) + align256((size_t)T * K * 4) + (size_t)T * K * PIMG;
  }
  return b;
}

int pfold_run(int nf, const PFoldDesc* d, void* ws, int* status, cudaStream_t s, int debug) {
  const int sms = num_sms();
  if (sms <= 0) return IFK_ERR_CUDA;
  if (nf > PFOLD_MAX_FOLDS) return IFK_ERR_SHAPE;
  PFBatch b;
  b.nf = 0;
  b.status = status;
  // a cross-CTA wait polls about every 0.1 us: 2^24 polls are a few seconds, the
  // test-only short limit (IFK_FOLD_DEBUG_WITHHOLD) a few milliseconds
  b.wait_limit = (debug & PFOLD_DEBUG_WITHHOLD) ? (1u << 14) : (1u << 24);
  b.withhold = (debug & PFOLD_DEBUG_WITHHOLD) ? 1 : 0;
  b.ctr = (int*)ws;
  b.abort_ = (int*)ws + 1;
  char* w = (char*)ws + 256;
  int tmax = 0, cbmax = 1, nsegs_total = 0, nconv = 0;
  const ConvGeo* convsrc[PFOLD_MAX_CONV] = {};
  for (int q = 0; q < nf; ++q) {  // flags first, so one memset clears them all
    const PFoldDesc& D = d[q];
    const int64_t T = pfold_subtiles(D);
    if (T <= 0) continue;
    if (D.nseg > MAX_SEGS || T > pfold_max_subtiles(D.n)) return IFK_ERR_SHAPE;  // callers split
    PFold& F = b.f[b.nf++];
    F.R = D.R;
    F.ldR = D.ldR;
    F.n = D.n;
    F.rows_R = D.rows_R;
    F.T = (int)T;
    F.K = (int)cdiv(F.n, NB);
    F.CB = (int)cdiv(F.n, WB);
    F.nseg = 0;
    F.seg0 = nsegs_total;
    int t0 = 0;
    int64_t off = 0;
    for (int g = 0; g < D.nseg; ++g) {
      const PFoldSeg& E = D.seg[g];
      if (E.rows <= 0) continue;
      if (E.tri && g + 1 < D.nseg) return IFK_ERR_SHAPE;  // only the last segment may be trapezoidal
      if (nsegs_total == PFOLD_MAX_BATCH_SEGS) return IFK_ERR_SHAPE;  // callers split
      PSeg& P = b.seg[nsegs_total++];
      ++F.nseg;
      P.X = E.X;
      P.ldX = E.ldX;
      P.rows = E.rows;
      P.row_off = off;
      P.ridx = E.ridx;
      P.src_rows = E.src_rows;
      P.cols = E.cols < 0 ? D.n : E.cols;
      P.t0 = t0;
      P.xkind = E.xkind;
      if (E.conv) {  // an im2col segment: its geometry goes to the launch's table
        int slot = -1;
        for (int q2 = 0; q2 < nconv; ++q2)
          if (memcmp(convsrc[q2], E.conv, sizeof(ConvGeo)) == 0) slot = q2;
        if (slot < 0) {
          if (nconv == PFOLD_MAX_CONV) return IFK_ERR_SHAPE;  // callers split
          slot = nconv;
          convsrc[nconv] = E.conv;
          b.conv[nconv++] = *E.conv;
        }
        P.xkind = XK_CONV + 2 * slot + (E.xkind == XK_BF16 ? 1 : 0);
      }
      P.tri = E.tri;
      P.ident = E.ident;
      t0 += (int)cdiv(E.rows, SUB);
      off += E.rows;
    }
    F.prog = (int*)w;
    w += align256((size_t)F.T * F.CB * 4);
    F.pflag = (int*)w;
    w += align256((size_t)F.T * F.K * 4);
    tmax = tmax > F.T ? tmax : F.T;
    cbmax = cbmax > F.CB ? cbmax : F.CB;
  }
  if (b.nf == 0) return IFK_OK;
  // the largest weight up to CBW_TARGET whose waves fit the table (at least
  // PIECE_CBW: every fold has at most pfold_max_subtiles sub-tiles)
  b.cbw = cbmax > 1 ? (int)mn<int64_t>(CBW_TARGET, (MAXW - tmax) / (cbmax - 1)) : CBW_TARGET;
  if (b.cbw < 1) return IFK_ERR_SHAPE;
  int maxw = 0;
  for (int g = 0; g < b.nf; ++g) {
    const int nw = num_waves(b.f[g].T, b.f[g].CB, b.cbw);
    maxw = maxw > nw ? maxw : nw;
  }
  const size_t flag_bytes = (size_t)(w - (char*)ws);
  for (int g = 0; g < b.nf; ++g) {
    b.f[g].img = (uint8_t*)w;
    w += (size_t)b.f[g].T * b.f[g].K * PIMG;
  }
  b.nwaves = maxw;
  int acc = 0;
  for (int dd = 0; dd < maxw; ++dd) {
    b.wave_off[dd] = acc;
    for (int g = 0; g < b.nf; ++g) {
      int tlo, cnt;
      wave_range(dd, b.f[g].T, b.f[g].CB, b.cbw, &tlo, &cnt);
      acc += cnt;
    }
  }
  b.wave_off[maxw] = acc;
  b.ntasks = acc;
  IFK_CUDA_TRY(cudaMemsetAsync(ws, 0, flag_bytes, s));
  const int grid = acc < sms ? acc : sms;
  fold_persistent_kernel<<<grid, TPB, SMEM, s>>>(b);
  IFK_CUDA_TRY(cudaGetLastError());
  return IFK_OK;
}

}  // namespace ifk
