// extern "C" entry points of libifk.so (declared in include/ifk.h).
// Host-side validation happens before anything is queued on the stream.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "ifk_common.cuh"
#include "ifk_internal.h"

using namespace ifk;

namespace {

constexpr size_t ALIGN = 256;
size_t align_up(size_t b) { return (b + ALIGN - 1) / ALIGN * ALIGN; }
bool aligned(const void* p) { return ((uintptr_t)p % ALIGN) == 0; }
bool dtype_ok(int d) { return d == IFK_F32 || d == IFK_BF16; }
bool prec_ok(int p) { return p == IFK_PREC_AUTO || p == IFK_PREC_FP32 || p == IFK_PREC_BF16; }
cudaStream_t S(ifk_stream_t s) { return (cudaStream_t)s; }

size_t wave_ws(int64_t rows, int64_t n) { return align_up(xw_bytes(rows, n)) + align_up(fold_tbuf_bytes(rows)); }
// persistent-fold workspace of one fold of `subtiles` sub-tiles (one launch takes at most
// pfold_max_subtiles of them; longer folds run as several launches over one workspace)
size_t pers_ws_subtiles(int64_t subtiles, int64_t n) {
  const int64_t t = std::min<int64_t>(subtiles, pfold_max_subtiles(n));
  return align_up(pfold_workspace(1, &t, &n));
}
size_t pers_ws(int64_t rows, int64_t n) { return pers_ws_subtiles(cdiv(rows, SUB), n); }
// per-fold workspace: enough for either schedule (fp32 waves or the persistent tensor-core fold)
size_t fold_ws(int64_t rows, int64_t n) { return std::max(wave_ws(rows, n), pers_ws(rows, n)); }

size_t elem_bytes(int xkind) { return xkind == 1 ? 2 : 4; }

// Cut a fold into launch pieces of at most pfold_max_subtiles sub-tiles and
// MAX_SEGS segments; piece i starts from the rows of the pieces before it.
int plan_pieces(const PFoldDesc& D, const PFoldSeg* segs, int nseg, std::vector<PFoldDesc>& out) {
  out.clear();
  const int64_t max_sub = pfold_max_subtiles(D.n);
  if (max_sub <= 0) return IFK_ERR_SHAPE;
  PFoldDesc cur = pfold_desc(D.R, D.ldR, D.n, D.rows_R);
  int64_t cur_sub = 0, done = 0;
  for (int g = 0; g < nseg; ++g) {
    const PFoldSeg& E = segs[g];
    if (E.rows <= 0) continue;
    if (E.tri && g + 1 < nseg) return IFK_ERR_SHAPE;  // only the last segment may be trapezoidal
    if (E.tri && cur.nseg > 0 && cdiv(E.rows, SUB) > max_sub - cur_sub) {
      // a trapezoidal chunk is not split: it starts the next launch
      out.push_back(cur);
      cur = pfold_desc(D.R, D.ldR, D.n, std::min<int64_t>(D.n, D.rows_R + done));
      cur_sub = 0;
    }
    int64_t off = 0;
    while (off < E.rows) {
      if (cur_sub == max_sub || cur.nseg == MAX_SEGS) {
        out.push_back(cur);
        cur = pfold_desc(D.R, D.ldR, D.n, std::min<int64_t>(D.n, D.rows_R + done));
        cur_sub = 0;
      }
      const int64_t take_sub = std::min<int64_t>(max_sub - cur_sub, cdiv(E.rows - off, SUB));
      const int64_t take = std::min<int64_t>(take_sub * SUB, E.rows - off);
      if (E.tri && take < E.rows) return IFK_ERR_SHAPE;  // trapezoidal chunks come in one piece
      PFoldSeg piece = E;
      piece.rows = take;
      if (E.ridx) piece.ridx = E.ridx + off;  // gathered rows: the index array advances
      else if (E.conv) piece.ldX = E.ldX + off;  // im2col rows: the first image row advances
      else if (E.xkind != 2) piece.X = (const char*)E.X + off * E.ldX * elem_bytes(E.xkind);
      cur.seg[cur.nseg++] = piece;
      cur_sub += take_sub;
      off += take;
      done += take;
    }
  }
  if (cur.nseg > 0) out.push_back(cur);
  return IFK_OK;
}

// Persistent tensor-core folds: groups of PFOLD_MAX_FOLDS folds share launches (a
// launch takes at most PFOLD_MAX_BATCH_SEGS segments; more go to a second launch);
// a fold longer than one launch allows continues in the group's next launch.  Fold f
// takes its segments from segs[f] (nsegs[f] of them) when segs is given, else
// from in[f].seg.
int run_persistent(int nf, const PFoldDesc* in, void* ws, int* status, cudaStream_t s,
                   const PFoldSeg* const* segs = nullptr, const int* nsegs = nullptr, int debug = 0) {
  for (int base = 0; base < nf; base += PFOLD_MAX_FOLDS) {
    const int cnt = std::min(PFOLD_MAX_FOLDS, nf - base);
    std::vector<std::vector<PFoldDesc>> pieces(cnt);
    size_t most = 0;
    for (int q = 0; q < cnt; ++q) {
      const PFoldDesc& D = in[base + q];
      const int rc = segs ? plan_pieces(D, segs[base + q], nsegs[base + q], pieces[q])
                          : plan_pieces(D, D.seg, D.nseg, pieces[q]);
      if (rc != IFK_OK) return rc;
      most = std::max(most, pieces[q].size());
    }
    for (size_t i = 0; i < most; ++i) {
      std::vector<PFoldDesc> d;
      int nseg = 0;
      std::vector<ConvGeo> geos;  // distinct im2col geometries of the launch being built
      auto new_geos = [&](const PFoldDesc& P) {
        int add = 0;
        for (int g = 0; g < P.nseg; ++g) {
          if (!P.seg[g].conv) continue;
          bool seen = false;
          for (const ConvGeo& c : geos) seen = seen || memcmp(&c, P.seg[g].conv, sizeof(ConvGeo)) == 0;
          for (int h = 0; h < g && !seen; ++h)
            seen = P.seg[h].conv && memcmp(P.seg[h].conv, P.seg[g].conv, sizeof(ConvGeo)) == 0;
          add += seen ? 0 : 1;
        }
        return add;
      };
      for (int q = 0; q < cnt; ++q) {
        if (i >= pieces[q].size()) continue;
        const PFoldDesc& P = pieces[q][i];
        if (!d.empty() && (nseg + P.nseg > PFOLD_MAX_BATCH_SEGS ||
                           (int)geos.size() + new_geos(P) > PFOLD_MAX_CONV)) {
          const int rc = pfold_run((int)d.size(), d.data(), ws, status, s, debug);
          if (rc != IFK_OK) return rc;
          d.clear();
          geos.clear();
          nseg = 0;
        }
        for (int g = 0; g < P.nseg; ++g) {
          if (!P.seg[g].conv) continue;
          bool seen = false;
          for (const ConvGeo& c : geos) seen = seen || memcmp(&c, P.seg[g].conv, sizeof(ConvGeo)) == 0;
          if (!seen) geos.push_back(*P.seg[g].conv);
        }
        d.push_back(P);
        nseg += P.nseg;
      }
      if (!d.empty()) {
        const int rc = pfold_run((int)d.size(), d.data(), ws, status, s, debug);
        if (rc != IFK_OK) return rc;
      }
    }
  }
  return IFK_OK;
}

}  // namespace

extern "C" {

const char* ifk_version(void) { return "ifkfac_b200 0.1.0 (sm_100a)"; }

const char* ifk_status_string(int status) {
  switch (status) {
    case IFK_OK: return "ok";
    case IFK_ERR_RANK: return "factor is rank deficient: fewer accumulated rows than columns";
    case IFK_ERR_NONFINITE: return "non-finite value in a factor";
    case IFK_ERR_SHAPE: return "inconsistent shape or leading dimension";
    case IFK_ERR_TIMEOUT: return "a bounded device-side wait timed out";
    case IFK_ERR_CUDA: return "CUDA runtime error";
    case IFK_ERR_WORKSPACE: return "workspace missing, too small or not 256-byte aligned";
    case IFK_ERR_DTYPE: return "unsupported element type";
    case IFK_ERR_ARG: return "invalid argument";
    case IFK_ERR_DEVICE: return "current device is not compute capability 10.0 (sm_100a)";
    case IFK_ERR_LIMIT: return "size above the fixed scratch of the no-allocation entry point";
    default: return "unknown status";
  }
}

int ifk_device_check(void) {
  int dev = 0, major = 0, minor = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return IFK_ERR_CUDA;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
    return IFK_ERR_CUDA;
  if (cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
    return IFK_ERR_CUDA;
  return (major == 10 && minor == 0) ? IFK_OK : IFK_ERR_DEVICE;
}

size_t ifk_tsqr_fold_workspace(int64_t rows, int64_t n) {
  if (rows < 0 || n <= 0) return 0;
  return fold_ws(rows, n);
}

int ifk_tsqr_fold(float* R, int64_t ldR, int64_t rows_R, const void* chunk, int64_t ld_chunk,
                  int64_t rows, int64_t n, int chunk_dtype, int prec, int flags, int* d_status,
                  void* workspace, size_t workspace_bytes, ifk_stream_t stream) {
  if (!R || (!chunk && rows > 0)) return IFK_ERR_ARG;
  if (n <= 0 || rows < 0 || rows_R < 0 || rows_R > n || ldR < n || (rows > 0 && ld_chunk < n))
    return IFK_ERR_SHAPE;
  if (!dtype_ok(chunk_dtype)) return IFK_ERR_DTYPE;
  if (!prec_ok(prec) || (flags & ~(IFK_FOLD_TRAPEZOIDAL_CHUNK | IFK_FOLD_DEBUG_WITHHOLD))) return IFK_ERR_ARG;
  if (rows == 0) return IFK_OK;
  if (!workspace || !aligned(workspace) || workspace_bytes < fold_ws(rows, n))
    return IFK_ERR_WORKSPACE;
  if (prec == IFK_PREC_AUTO) prec = chunk_dtype == IFK_BF16 ? IFK_PREC_BF16 : IFK_PREC_FP32;
  if ((flags & IFK_FOLD_DEBUG_WITHHOLD) && prec != IFK_PREC_BF16) return IFK_ERR_ARG;
  if (prec == IFK_PREC_BF16) {
    PFoldDesc d = pfold_desc(R, ldR, n, rows_R);
    pfold_add(d, chunk, ld_chunk, rows, chunk_dtype == IFK_BF16 ? 1 : 0, 0.f,
              (flags & IFK_FOLD_TRAPEZOIDAL_CHUNK) ? 1 : 0);
    return run_persistent(1, &d, workspace, d_status, S(stream), nullptr, nullptr,
                          (flags & IFK_FOLD_DEBUG_WITHHOLD) ? PFOLD_DEBUG_WITHHOLD : 0);
  }
  FoldArgs a;
  a.R = R;
  a.ldR = ldR;
  a.X = (float*)workspace;
  a.ldX = xw_ld(n);
  a.Tb = (float*)((char*)workspace + align_up(xw_bytes(rows, n)));
  a.n = n;
  a.rows = rows;
  a.rows_R = rows_R;
  a.tiles = (int)cdiv(rows, SUB);
  a.K = (int)cdiv(n, NB);
  a.tri = (flags & IFK_FOLD_TRAPEZOIDAL_CHUNK) ? 1 : 0;
  a.err = d_status;
  cudaStream_t s = S(stream);
  int rc = copy_chunk(a.X, a.ldX, chunk, ld_chunk, rows, n, chunk_dtype, s);
  if (rc != IFK_OK) return rc;
  return fold_run(a, prec, s);
}

size_t ifk_tsqr_fold_batched_workspace(int nfolds, const int64_t* rows, const int64_t* n) {
  if (nfolds <= 0 || !rows || !n) return 0;
  size_t b = 0;
  for (int f = 0; f < nfolds; ++f)
    if (rows[f] > 0 && n[f] > 0) b += fold_ws(rows[f], n[f]);
  return b;
}

int ifk_tsqr_fold_batched(int nfolds, float* const* R, const int64_t* ldR, const int64_t* rows_R,
                          const void* const* chunk, const int64_t* ld_chunk, const int64_t* rows,
                          const int64_t* n, int chunk_dtype, int prec, int flags, int* d_status,
                          void* workspace, size_t workspace_bytes, ifk_stream_t stream) {
  if (nfolds < 0 || (nfolds > 0 && (!R || !ldR || !rows_R || !chunk || !ld_chunk || !rows || !n)))
    return IFK_ERR_ARG;
  if (!dtype_ok(chunk_dtype)) return IFK_ERR_DTYPE;
  if (!prec_ok(prec) || (flags & ~IFK_FOLD_TRAPEZOIDAL_CHUNK)) return IFK_ERR_ARG;
  for (int f = 0; f < nfolds; ++f) {
    if (!R[f] || (!chunk[f] && rows[f] > 0)) return IFK_ERR_ARG;
    if (n[f] <= 0 || rows[f] < 0 || rows_R[f] < 0 || rows_R[f] > n[f] || ldR[f] < n[f] ||
        (rows[f] > 0 && ld_chunk[f] < n[f]))
      return IFK_ERR_SHAPE;
  }
  if (!workspace || !aligned(workspace) ||
      workspace_bytes < ifk_tsqr_fold_batched_workspace(nfolds, rows, n))
    return IFK_ERR_WORKSPACE;
  if (prec == IFK_PREC_AUTO) prec = chunk_dtype == IFK_BF16 ? IFK_PREC_BF16 : IFK_PREC_FP32;
  cudaStream_t s = S(stream);
  if (prec == IFK_PREC_BF16) {
    std::vector<PFoldDesc> d;
    for (int f = 0; f < nfolds; ++f) {
      if (rows[f] == 0) continue;
      d.push_back(pfold_desc(R[f], ldR[f], n[f], rows_R[f]));
      pfold_add(d.back(), chunk[f], ld_chunk[f], rows[f], chunk_dtype == IFK_BF16 ? 1 : 0, 0.f,
                (flags & IFK_FOLD_TRAPEZOIDAL_CHUNK) ? 1 : 0);
    }
    return d.empty() ? IFK_OK : run_persistent((int)d.size(), d.data(), workspace, d_status, s);
  }
  char* ws = (char*)workspace;
  FoldBatch b;
  b.nf = 0;
  for (int f = 0; f < nfolds; ++f) {
    if (rows[f] == 0) continue;
    FoldArgs& a = b.f[b.nf++];
    a.R = R[f];
    a.ldR = ldR[f];
    a.X = (float*)ws;
    a.ldX = xw_ld(n[f]);
    a.Tb = (float*)(ws + align_up(xw_bytes(rows[f], n[f])));
    ws += fold_ws(rows[f], n[f]);
    a.n = n[f];
    a.rows = rows[f];
    a.rows_R = rows_R[f];
    a.tiles = (int)cdiv(rows[f], SUB);
    a.K = (int)cdiv(n[f], NB);
    a.tri = (flags & IFK_FOLD_TRAPEZOIDAL_CHUNK) ? 1 : 0;
    a.err = d_status;
    int rc = copy_chunk(a.X, a.ldX, chunk[f], ld_chunk[f], rows[f], n[f], chunk_dtype, s);
    if (rc != IFK_OK) return rc;
    if (b.nf == MAX_FOLDS) {
      rc = fold_run_batch(b, prec, s);
      if (rc != IFK_OK) return rc;
      b.nf = 0;
    }
  }
  return fold_run_batch(b, prec, s);
}

// fp32 wave fold of one chunk (copied into the workspace) or of ident * I when chunk is null
static int fold_fp32(float* R, int64_t ldR, int64_t rows_R, const void* chunk, int64_t ld_chunk,
                     int64_t rows, int64_t n, int chunk_dtype, int tri, float ident, int prec,
                     int* d_status, void* workspace, cudaStream_t s, const int64_t* ridx = nullptr,
                     int64_t src_rows = 0, int64_t cols = -1, const ConvGeo* conv = nullptr) {
  FoldArgs a;
  a.R = R;
  a.ldR = ldR;
  a.X = (float*)workspace;
  a.ldX = xw_ld(n);
  a.Tb = (float*)((char*)workspace + align_up(xw_bytes(rows, n)));
  a.n = n;
  a.rows = rows;
  a.rows_R = rows_R;
  a.tiles = (int)cdiv(rows, SUB);
  a.K = (int)cdiv(n, NB);
  a.tri = tri;
  a.err = d_status;
  const int rc = chunk ? copy_chunk(a.X, a.ldX, chunk, ld_chunk, rows, n, chunk_dtype, s, ridx, src_rows, cols,
                                    d_status, conv)
                       : fill_scaled_identity(a.X, a.ldX, n, ident, s);
  if (rc != IFK_OK) return rc;
  return fold_run(a, prec, s);
}

// im2col geometry of a segment (checked), or false when it is not a valid one
static bool conv_geo(const ifk_segment& E, ConvGeo* g) {
  const ifk_conv2d* c = E.conv;
  if (c->batch <= 0 || c->channels <= 0 || c->height <= 0 || c->width <= 0 || c->kernel_h <= 0 ||
      c->kernel_w <= 0 || c->stride_h <= 0 || c->stride_w <= 0 || c->pad_h < 0 || c->pad_w < 0 ||
      c->dilation_h <= 0 || c->dilation_w <= 0)
    return false;
  const int64_t ho = (c->height + 2 * c->pad_h - c->dilation_h * (c->kernel_h - 1) - 1) / c->stride_h + 1;
  const int64_t wo = (c->width + 2 * c->pad_w - c->dilation_w * (c->kernel_w - 1) - 1) / c->stride_w + 1;
  if (ho <= 0 || wo <= 0 || ho > (1 << 30) || wo > (1 << 30)) return false;
  g->B = c->batch;
  g->C = c->channels;
  g->H = c->height;
  g->W = c->width;
  g->kh = c->kernel_h;
  g->kw = c->kernel_w;
  g->sh = c->stride_h;
  g->sw = c->stride_w;
  g->ph = c->pad_h;
  g->pw = c->pad_w;
  g->dh = c->dilation_h;
  g->dw = c->dilation_w;
  g->Ho = (int)ho;
  g->Wo = (int)wo;
  return true;
}

static int64_t seg_base(int f, const int* nseg) {
  int64_t b = 0;
  for (int g = 0; g < f; ++g) b += nseg[g];
  return b;
}

size_t ifk_tsqr_fold_segments_workspace(int nfolds, const int64_t* n, const int* nseg,
                                        const ifk_segment* segs, const double* ident_tail) {
  if (nfolds <= 0 || !n || !nseg) return 0;
  size_t b = 0;
  for (int f = 0; f < nfolds; ++f) {
    if (n[f] <= 0 || nseg[f] < 0 || (nseg[f] > 0 && !segs)) return 0;
    const int64_t base = seg_base(f, nseg);
    int64_t sub = 0, most = 0;
    for (int g = 0; g < nseg[f]; ++g) {
      const int64_t r = std::max<int64_t>(segs[base + g].rows, 0);
      sub += cdiv(r, SUB);
      most = std::max(most, r);
    }
    if (ident_tail && ident_tail[f] > 0) {
      sub += cdiv(n[f], SUB);
      most = std::max(most, n[f]);
    }
    if (sub > 0) b += std::max(pers_ws_subtiles(sub, n[f]), wave_ws(std::max<int64_t>(most, 1), n[f]));
  }
  return b;
}

// Rows of fold f's segments in total, and whether they can share one fp32 wave
// schedule with the sub-tile sequence of one fold per segment in turn: every
// segment but the last with rows holds a multiple of SUB rows.
static bool fp32_concat_rows(int f, const int* nseg, const ifk_segment* segs, int64_t* total) {
  const int64_t base = seg_base(f, nseg);
  int64_t t = 0;
  int last = -1;
  for (int g = 0; g < nseg[f]; ++g)
    if (segs[base + g].rows > 0) last = g;
  bool ok = true;
  for (int g = 0; g < nseg[f]; ++g) {
    const int64_t r = std::max<int64_t>(segs[base + g].rows, 0);
    if (r > 0 && g != last && r % SUB != 0) ok = false;
    t += r;
  }
  *total = t;
  return ok;
}

size_t ifk_tsqr_fold_segments_fp32_workspace(int nfolds, const int64_t* n, const int* nseg,
                                             const ifk_segment* segs, const double* ident_tail) {
  const size_t base = ifk_tsqr_fold_segments_workspace(nfolds, n, nseg, segs, ident_tail);
  if (base == 0) return 0;
  size_t b = 0;
  for (int f = 0; f < nfolds; ++f) {
    int64_t total = 0;
    fp32_concat_rows(f, nseg, segs, &total);
    const int64_t rows = std::max<int64_t>(total, (ident_tail && ident_tail[f] > 0) ? n[f] : 0);
    if (rows > 0) b += wave_ws(rows, n[f]);
  }
  return std::max(base, b);
}

int ifk_tsqr_fold_segments(int nfolds, float* const* R, const int64_t* ldR, const int64_t* rows_R,
                           const int64_t* n, const int* nseg, const ifk_segment* segs, int chunk_dtype,
                           const double* ident_tail, int prec, int* d_status, void* workspace,
                           size_t workspace_bytes, ifk_stream_t stream) {
  if (nfolds < 0 || (nfolds > 0 && (!R || !ldR || !rows_R || !n || !nseg))) return IFK_ERR_ARG;
  const bool per_seg = chunk_dtype == IFK_PER_SEGMENT_DTYPE;
  if (!dtype_ok(chunk_dtype) && !per_seg) return IFK_ERR_DTYPE;
  if (!prec_ok(prec) || (per_seg && prec == IFK_PREC_AUTO)) return IFK_ERR_ARG;
  bool any = false;
  for (int f = 0; f < nfolds; ++f) {
    if (!R[f] || nseg[f] < 0 || (nseg[f] > 0 && !segs)) return IFK_ERR_ARG;
    if (n[f] <= 0 || rows_R[f] < 0 || rows_R[f] > n[f] || ldR[f] < n[f]) return IFK_ERR_SHAPE;
    if (ident_tail && !(ident_tail[f] >= 0)) return IFK_ERR_ARG;
    const int64_t base = seg_base(f, nseg);
    for (int g = 0; g < nseg[f]; ++g) {
      const ifk_segment& E = segs[base + g];
      if (E.rows < 0) return IFK_ERR_SHAPE;
      if (E.rows == 0) continue;
      if (!E.chunk) return IFK_ERR_ARG;
      if (E.cols != n[f] && E.cols != n[f] - 1) return IFK_ERR_SHAPE;
      if (E.conv) {
        // an NCHW image read through im2col: C kh kw columns, B Ho Wo image rows
        ConvGeo g;
        if (!conv_geo(E, &g)) return IFK_ERR_SHAPE;
        if (E.cols != g.C * g.kh * g.kw || E.src_rows != g.B * g.Ho * g.Wo) return IFK_ERR_SHAPE;
        if (!E.row_index && E.rows > E.src_rows) return IFK_ERR_SHAPE;
      } else {
        if (E.cols < 1 || E.ld < E.cols) return IFK_ERR_SHAPE;
        if (E.row_index && E.src_rows <= 0) return IFK_ERR_SHAPE;
      }
      if (per_seg && !dtype_ok(E.dtype)) return IFK_ERR_DTYPE;
      any = true;
    }
    any = any || (ident_tail && ident_tail[f] > 0);
  }
  if (!any) return IFK_OK;
  if (!workspace || !aligned(workspace) ||
      workspace_bytes < ifk_tsqr_fold_segments_workspace(nfolds, n, nseg, segs, ident_tail))
    return IFK_ERR_WORKSPACE;
  if (prec == IFK_PREC_AUTO) prec = chunk_dtype == IFK_BF16 ? IFK_PREC_BF16 : IFK_PREC_FP32;
  cudaStream_t s = S(stream);
  // im2col geometries, one per segment that has one (stable storage for the launcher)
  int64_t nsegs = 0;
  for (int f = 0; f < nfolds; ++f) nsegs += nseg[f];
  std::vector<ConvGeo> geo((size_t)nsegs);
  for (int64_t i = 0; i < nsegs; ++i)
    if (segs[i].conv && segs[i].rows > 0) conv_geo(segs[i], &geo[(size_t)i]);
  if (prec == IFK_PREC_BF16) {
    std::vector<PFoldDesc> d((size_t)nfolds);
    std::vector<std::vector<PFoldSeg>> sg((size_t)nfolds);
    std::vector<const PFoldSeg*> sp((size_t)nfolds);
    std::vector<int> ns((size_t)nfolds);
    for (int f = 0; f < nfolds; ++f) {
      d[f] = pfold_desc(R[f], ldR[f], n[f], rows_R[f]);
      const int64_t base = seg_base(f, nseg);
      for (int g = 0; g < nseg[f]; ++g) {
        const ifk_segment& E = segs[base + g];
        if (E.rows <= 0) continue;
        PFoldSeg P;
        P.X = E.chunk;
        P.ldX = E.conv ? 0 : E.ld;  // im2col segments: the first image row
        P.rows = E.rows;
        P.xkind = (per_seg ? E.dtype : chunk_dtype) == IFK_BF16 ? 1 : 0;
        P.ident = 0.f;
        P.tri = 0;
        P.ridx = E.row_index;
        P.src_rows = E.src_rows;
        P.cols = E.cols;
        P.conv = E.conv ? &geo[(size_t)(base + g)] : nullptr;
        sg[f].push_back(P);
      }
      if (ident_tail && ident_tail[f] > 0) {
        PFoldSeg P;
        P.X = nullptr;
        P.ldX = 0;
        P.rows = n[f];
        P.xkind = 2;
        P.ident = (float)ident_tail[f];
        P.tri = 1;
        sg[f].push_back(P);
      }
      sp[f] = sg[f].data();
      ns[f] = (int)sg[f].size();
    }
    // folds without rows are dropped by the launcher
    return run_persistent(nfolds, d.data(), workspace, d_status, s, sp.data(), ns.data());
  }
  // fp32 mode.  When every fold's segments can be concatenated (see
  // fp32_concat_rows) and the workspace covers the concatenation, the segments of
  // each fold are copied one after another into its part of the workspace and all
  // folds run one wave schedule together: T + K - 1 waves instead of one schedule
  // per segment, with the same sub-tile sequence; the identity tails follow as one
  // more schedule of trapezoidal folds.
  {
    bool concat = nfolds <= MAX_FOLDS;
    size_t need = 0;
    std::vector<int64_t> tot((size_t)std::max(nfolds, 0));
    for (int f = 0; f < nfolds && concat; ++f) {
      concat = fp32_concat_rows(f, nseg, segs, &tot[(size_t)f]);
      const int64_t rows = std::max<int64_t>(tot[(size_t)f], (ident_tail && ident_tail[f] > 0) ? n[f] : 0);
      if (rows > 0) need += wave_ws(rows, n[f]);
    }
    if (concat && workspace_bytes >= need) {
      std::vector<char*> wsf((size_t)nfolds);
      char* w = (char*)workspace;
      for (int f = 0; f < nfolds; ++f) {
        wsf[(size_t)f] = w;
        const int64_t rows = std::max<int64_t>(tot[(size_t)f], (ident_tail && ident_tail[f] > 0) ? n[f] : 0);
        if (rows > 0) w += wave_ws(rows, n[f]);
      }
      auto args = [&](int f, int64_t rows, int64_t rr, int tri) {
        FoldArgs a;
        a.R = R[f];
        a.ldR = ldR[f];
        a.X = (float*)wsf[(size_t)f];
        a.ldX = xw_ld(n[f]);
        a.Tb = (float*)(wsf[(size_t)f] + align_up(xw_bytes(rows, n[f])));
        a.n = n[f];
        a.rows = rows;
        a.rows_R = rr;
        a.tiles = (int)cdiv(rows, SUB);
        a.K = (int)cdiv(n[f], NB);
        a.tri = tri;
        a.err = d_status;
        return a;
      };
      FoldBatch b;
      b.nf = 0;
      for (int f = 0; f < nfolds; ++f) {
        if (tot[(size_t)f] == 0) continue;
        FoldArgs a = args(f, tot[(size_t)f], rows_R[f], 0);
        const int64_t base = seg_base(f, nseg);
        int64_t off = 0;
        for (int g = 0; g < nseg[f]; ++g) {
          const ifk_segment& E = segs[base + g];
          if (E.rows <= 0) continue;
          const int rc = copy_chunk(a.X + off * a.ldX, a.ldX, E.chunk, E.ld, E.rows, n[f],
                                    per_seg ? E.dtype : chunk_dtype, s, E.row_index, E.src_rows, E.cols, d_status,
                                    E.conv ? &geo[(size_t)(base + g)] : nullptr);
          if (rc != IFK_OK) return rc;
          off += E.rows;
        }
        b.f[b.nf++] = a;
      }
      int rc = fold_run_batch(b, prec, s);
      if (rc != IFK_OK) return rc;
      b.nf = 0;
      for (int f = 0; f < nfolds; ++f) {
        if (!(ident_tail && ident_tail[f] > 0)) continue;
        FoldArgs a = args(f, n[f], std::min<int64_t>(n[f], rows_R[f] + tot[(size_t)f]), 1);
        rc = fill_scaled_identity(a.X, a.ldX, n[f], (float)ident_tail[f], s);
        if (rc != IFK_OK) return rc;
        b.f[b.nf++] = a;
      }
      return fold_run_batch(b, prec, s);
    }
  }
  // otherwise the segments of each fold one after another through the wave schedule
  for (int f = 0; f < nfolds; ++f) {
    int64_t rr = rows_R[f];
    const int64_t base = seg_base(f, nseg);
    for (int g = 0; g < nseg[f]; ++g) {
      const ifk_segment& E = segs[base + g];
      if (E.rows == 0) continue;
      const int rc = fold_fp32(R[f], ldR[f], rr, E.chunk, E.ld, E.rows, n[f], per_seg ? E.dtype : chunk_dtype, 0, 0.f,
                               prec, d_status, workspace, s, E.row_index, E.src_rows, E.cols,
                               E.conv ? &geo[(size_t)(base + g)] : nullptr);
      if (rc != IFK_OK) return rc;
      rr = std::min<int64_t>(n[f], rr + E.rows);
    }
    if (ident_tail && ident_tail[f] > 0) {
      const int rc = fold_fp32(R[f], ldR[f], rr, nullptr, 0, n[f], n[f], IFK_F32, 1, (float)ident_tail[f], prec,
                               d_status, workspace, s);
      if (rc != IFK_OK) return rc;
    }
  }
  return IFK_OK;
}

// ---- R-tree merge of factors held by one process ----------------------------

size_t ifk_rtree_merge_workspace(int nfactors, int64_t n) {
  if (nfactors <= 0 || n <= 0) return 0;
  // the widest round merges nfactors / 2 pairs, each a fold of up to n rows
  return std::max<size_t>((size_t)(nfactors / 2) * fold_ws(n, n), ALIGN);
}

int ifk_rtree_merge(int nfactors, float* const* R, const int64_t* ldR, const int64_t* rows, int64_t n, int prec,
                    int64_t* rows_out, int* d_status, void* workspace, size_t workspace_bytes,
                    ifk_stream_t stream) {
  if (nfactors <= 0 || !R || !ldR || !rows || !rows_out) return IFK_ERR_ARG;
  if (!prec_ok(prec) || prec == IFK_PREC_AUTO) return IFK_ERR_ARG;
  if (n <= 0) return IFK_ERR_SHAPE;
  for (int i = 0; i < nfactors; ++i) {
    if (!R[i]) return IFK_ERR_ARG;
    if (ldR[i] < n || rows[i] < 0 || rows[i] > n) return IFK_ERR_SHAPE;
  }
  if (nfactors > 1 && (!workspace || !aligned(workspace) ||
                       workspace_bytes < ifk_rtree_merge_workspace(nfactors, n)))
    return IFK_ERR_WORKSPACE;
  // items of the current round: (factor index, meaningful rows)
  std::vector<std::pair<int, int64_t>> items;
  for (int i = 0; i < nfactors; ++i) items.emplace_back(i, rows[i]);
  while (items.size() > 1) {
    std::vector<std::pair<int, int64_t>> next;
    std::vector<float*> ra;
    std::vector<const void*> rb;
    std::vector<int64_t> lda, ldb, rows_a, rows_b, nn;
    for (size_t i = 0; i < items.size(); i += 2) {
      if (i + 1 == items.size()) {  // odd one out: carried forward
        next.push_back(items[i]);
        continue;
      }
      const auto a = items[i], b = items[i + 1];
      next.emplace_back(a.first, std::min<int64_t>(n, a.second + b.second));
      if (b.second == 0) continue;
      ra.push_back(R[a.first]);
      lda.push_back(ldR[a.first]);
      rows_a.push_back(a.second);
      rb.push_back(R[b.first]);
      ldb.push_back(ldR[b.first]);
      // bf16 mode: rows past a factor's count stay zero (the fold's rank bound), so
      // only the meaningful rows are folded; fp32 mode folds the whole factor, where
      // a zero pivot can leave content below that count
      rows_b.push_back(prec == IFK_PREC_BF16 ? b.second : n);
      nn.push_back(n);
    }
    if (!ra.empty()) {
      // the merges of one round share one launch (each a trapezoidal-chunk fold)
      const int rc = ifk_tsqr_fold_batched((int)ra.size(), ra.data(), lda.data(), rows_a.data(), rb.data(),
                                           ldb.data(), rows_b.data(), nn.data(), IFK_F32, prec,
                                           IFK_FOLD_TRAPEZOIDAL_CHUNK, d_status, workspace, workspace_bytes,
                                           stream);
      if (rc != IFK_OK) return rc;
    }
    items.swap(next);
  }
  *rows_out = items[0].second;
  return IFK_OK;
}

size_t ifk_finalize_workspace(int64_t n) {
  if (n <= 0) return 0;
  return align_up((size_t)n * xw_ld(n) * sizeof(float)) + fold_ws(n, n);
}

int ifk_finalize(const float* R_in, int64_t ldR, int64_t rows_R, int64_t n, double rows_total,
                 double damping, void* R_out, int64_t ld_out, int out_dtype, int prec,
                 int* d_status, void* workspace, size_t workspace_bytes, ifk_stream_t stream) {
  if (!R_in || !R_out) return IFK_ERR_ARG;
  if (n <= 0 || ldR < n || ld_out < n) return IFK_ERR_SHAPE;
  if (!dtype_ok(out_dtype)) return IFK_ERR_DTYPE;
  if (!prec_ok(prec) || !(rows_total > 0) || !(damping >= 0)) return IFK_ERR_ARG;
  if (rows_R < n) return IFK_ERR_RANK;
  if (!workspace || !aligned(workspace) || workspace_bytes < ifk_finalize_workspace(n))
    return IFK_ERR_WORKSPACE;
  if (prec == IFK_PREC_AUTO) prec = out_dtype == IFK_BF16 ? IFK_PREC_BF16 : IFK_PREC_FP32;
  cudaStream_t s = S(stream);
  const int64_t ldF = xw_ld(n);
  float* Rf = (float*)workspace;
  void* fws = (char*)workspace + align_up((size_t)n * ldF * sizeof(float));
  if (damping == 0)  // nothing to fold: scale, cast and check in one pass
    return finish_factor(R_out, ld_out, out_dtype, R_in, ldR, n, d_status, s, (float)std::sqrt(rows_total));
  int rc = scale_upper(Rf, ldF, R_in, ldR, n, (float)std::sqrt(rows_total), s);
  if (rc != IFK_OK) return rc;
  if (damping > 0 && prec == IFK_PREC_BF16) {
    PFoldDesc d = pfold_desc(Rf, ldF, n, n);
    pfold_add(d, nullptr, 0, n, 2, (float)std::sqrt(damping), 1);
    rc = run_persistent(1, &d, fws, d_status, s);
    if (rc != IFK_OK) return rc;
  } else if (damping > 0) {
    FoldArgs a;
    a.R = Rf;
    a.ldR = ldF;
    a.X = (float*)fws;
    a.ldX = xw_ld(n);
    a.Tb = (float*)((char*)fws + align_up(xw_bytes(n, n)));
    a.n = n;
    a.rows = n;
    a.rows_R = n;
    a.tiles = (int)cdiv(n, SUB);
    a.K = (int)cdiv(n, NB);
    a.tri = 1;
    a.err = d_status;
    rc = fill_scaled_identity(a.X, a.ldX, n, (float)std::sqrt(damping), s);
    if (rc != IFK_OK) return rc;
    rc = fold_run(a, prec, s);
    if (rc != IFK_OK) return rc;
  }
  return finish_factor(R_out, ld_out, out_dtype, Rf, ldF, n, d_status, s);
}

size_t ifk_finalize_batched_workspace(int nfactors, const int64_t* n) {
  if (nfactors <= 0 || !n) return 0;
  size_t b = 0;
  for (int f = 0; f < nfactors; ++f)
    if (n[f] > 0) b += ifk_finalize_workspace(n[f]);
  return b;
}

}  // extern "C"

static int finalize_many(int nfactors, const float* const* R_in, const int64_t* ldR, const int64_t* rows_R,
                         const int64_t* n, const double* rows_total, double damping, void* const* R_out,
                         const int64_t* ld_out, int out_dtype, int prec, int* d_status, int* const* f_status,
                         void* workspace, size_t workspace_bytes, ifk_stream_t stream) {
  if (nfactors < 0 ||
      (nfactors > 0 && (!R_in || !ldR || !rows_R || !n || !rows_total || !R_out || !ld_out)))
    return IFK_ERR_ARG;
  if (!dtype_ok(out_dtype)) return IFK_ERR_DTYPE;
  if (!prec_ok(prec) || !(damping >= 0)) return IFK_ERR_ARG;
  for (int f = 0; f < nfactors; ++f) {
    if (!R_in[f] || !R_out[f] || !(rows_total[f] > 0)) return IFK_ERR_ARG;
    if (n[f] <= 0 || ldR[f] < n[f] || ld_out[f] < n[f]) return IFK_ERR_SHAPE;
    if (rows_R[f] < n[f]) return IFK_ERR_RANK;
  }
  if (!workspace || !aligned(workspace) ||
      workspace_bytes < ifk_finalize_batched_workspace(nfactors, n))
    return IFK_ERR_WORKSPACE;
  if (prec == IFK_PREC_AUTO) prec = out_dtype == IFK_BF16 ? IFK_PREC_BF16 : IFK_PREC_FP32;
  cudaStream_t s = S(stream);
  // workspace: [fp32 copies of up to MAX_FOLDS factors | one fold area], reused per group
  for (int base = 0; base < nfactors; base += MAX_FOLDS) {
    const int cnt = std::min(MAX_FOLDS, nfactors - base);
    char* ws = (char*)workspace;
    float* Rf[MAX_FOLDS];
    if (damping == 0) {
      // nothing to fold: each factor is scaled, cast and checked in one pass
      for (int q = 0; q < cnt; ++q) {
        const int f = base + q;
        int* st = f_status ? f_status[f] : d_status;
        const int rc = finish_factor(R_out[f], ld_out[f], out_dtype, R_in[f], ldR[f], n[f], st, s,
                                     (float)std::sqrt(rows_total[f]));
        if (rc != IFK_OK) return rc;
      }
      continue;
    }
    for (int q = 0; q < cnt; ++q) {
      const int f = base + q;
      Rf[q] = (float*)ws;
      ws += align_up((size_t)n[f] * xw_ld(n[f]) * sizeof(float));
      int rc = scale_upper(Rf[q], xw_ld(n[f]), R_in[f], ldR[f], n[f], (float)std::sqrt(rows_total[f]), s);
      if (rc != IFK_OK) return rc;
    }
    if (damping > 0) {
      int rc;
      if (prec == IFK_PREC_BF16) {
        PFoldDesc pd[MAX_FOLDS];
        for (int q = 0; q < cnt; ++q) {
          const int f = base + q;
          pd[q] = pfold_desc(Rf[q], xw_ld(n[f]), n[f], n[f]);
          pfold_add(pd[q], nullptr, 0, n[f], 2, (float)std::sqrt(damping), 1);
        }
        // a timed-out wait of the shared launch is reported to the group's first factor
        rc = run_persistent(cnt, pd, ws, d_status ? d_status : (f_status ? f_status[base] : nullptr), s);
      } else {
        FoldBatch b;
        b.nf = 0;
        char* fw = ws;
        for (int q = 0; q < cnt; ++q) {
          const int f = base + q;
          FoldArgs& a = b.f[b.nf++];
          a.R = Rf[q];
          a.ldR = xw_ld(n[f]);
          a.X = (float*)fw;
          a.ldX = xw_ld(n[f]);
          a.Tb = (float*)(fw + align_up(xw_bytes(n[f], n[f])));
          fw += fold_ws(n[f], n[f]);
          a.n = n[f];
          a.rows = n[f];
          a.rows_R = n[f];
          a.tiles = (int)cdiv(n[f], SUB);
          a.K = (int)cdiv(n[f], NB);
          a.tri = 1;
          a.err = f_status ? f_status[f] : d_status;
          rc = fill_scaled_identity(a.X, a.ldX, n[f], (float)std::sqrt(damping), s);
          if (rc != IFK_OK) return rc;
        }
        rc = fold_run_batch(b, prec, s);
      }
      if (rc != IFK_OK) return rc;
    }
    for (int q = 0; q < cnt; ++q) {
      const int f = base + q;
      int* st = f_status ? f_status[f] : d_status;
      const int rc = finish_factor(R_out[f], ld_out[f], out_dtype, Rf[q], xw_ld(n[f]), n[f], st, s);
      if (rc != IFK_OK) return rc;
    }
  }
  return IFK_OK;
}

namespace {

int pad_grid(int64_t total) { return (int)std::min<int64_t>(cdiv(total, 256), 4096); }

size_t natgrad_persist_bytes(int64_t n_out, int64_t n_in) {
  return align_up(trsm_persist_inverse_bytes(n_out)) + align_up(trsm_persist_inverse_bytes(n_in)) +
         align_up(std::max(trsm_persist_workspace(n_out, n_in), trsm_persist_workspace(n_in, n_out)));
}

// Orders that are not multiples of 8 (the persistent solves copy 16-byte rows):
// the solves run on [[R, 0], [0, I]] of order pad8(n) and a zero-padded right-hand
// side, which leave the leading block exactly as the unpadded solves define it.
int64_t pad8(int64_t n) { return (n + 7) / 8 * 8; }
bool needs_pad(int64_t n_out, int64_t n_in) { return n_out % 8 != 0 || n_in % 8 != 0; }
// the padded copies after the persistent area of the padded orders:
// R_G' | R_X' (bf16) | B' (fp32, p_out x p_in) | b' (fp32, p_out)
size_t pad_copies_bytes(int64_t n_out, int64_t n_in) {
  const int64_t po = pad8(n_out), pi = pad8(n_in);
  return align_up((size_t)po * po * 2) + align_up((size_t)pi * pi * 2) + align_up((size_t)po * pi * 4) +
         align_up((size_t)po * 4);
}
size_t padded_natgrad_bytes(int64_t n_out, int64_t n_in) {
  return align_up(natgrad_persist_bytes(pad8(n_out), pad8(n_in))) + pad_copies_bytes(n_out, n_in);
}

__global__ void pad_factor_kernel(const __nv_bfloat16* R, int64_t ld, int64_t n, __nv_bfloat16* P, int64_t np) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < np * np; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / np, c = i % np;
    P[i] = (r < n && c < n) ? R[r * ld + c] : __float2bfloat16(r == c ? 1.f : 0.f);
  }
}

struct Padded {
  __nv_bfloat16 *Rg, *Rx;
  float *B, *b;
  uint8_t *inv_g, *inv_x, *scratch;
  int64_t po, pi;
};
// Lay the padded problem out in ws and fill it: factors, zero-padded gradient (and bias).
int pad_problem(uint8_t* ws, const void* R_G, int64_t ld_rg, const void* R_X, int64_t ld_rx, const float* g,
                int64_t ld_g, const float* gb, int64_t n_out, int64_t n_in, Padded& P, cudaStream_t s) {
  P.po = pad8(n_out);
  P.pi = pad8(n_in);
  P.inv_g = ws;
  P.inv_x = P.inv_g + align_up(trsm_persist_inverse_bytes(P.po));
  P.scratch = P.inv_x + align_up(trsm_persist_inverse_bytes(P.pi));
  uint8_t* q = ws + align_up(natgrad_persist_bytes(P.po, P.pi));
  P.Rg = (__nv_bfloat16*)q;
  q += align_up((size_t)P.po * P.po * 2);
  P.Rx = (__nv_bfloat16*)q;
  q += align_up((size_t)P.pi * P.pi * 2);
  P.B = (float*)q;
  q += align_up((size_t)P.po * P.pi * 4);
  P.b = (float*)q;
  pad_factor_kernel<<<pad_grid(P.po * P.po), 256, 0, s>>>((const __nv_bfloat16*)R_G, ld_rg, n_out, P.Rg, P.po);
  pad_factor_kernel<<<pad_grid(P.pi * P.pi), 256, 0, s>>>((const __nv_bfloat16*)R_X, ld_rx, n_in, P.Rx, P.pi);
  IFK_CUDA_TRY(cudaGetLastError());
  IFK_CUDA_TRY(cudaMemsetAsync(P.B, 0, (size_t)P.po * P.pi * 4, s));
  IFK_CUDA_TRY(cudaMemcpy2DAsync(P.B, P.pi * sizeof(float), g, ld_g * sizeof(float), n_in * sizeof(float), n_out,
                                 cudaMemcpyDeviceToDevice, s));
  if (gb) {
    IFK_CUDA_TRY(cudaMemsetAsync(P.b, 0, (size_t)P.po * 4, s));
    IFK_CUDA_TRY(cudaMemcpyAsync(P.b, gb, n_out * sizeof(float), cudaMemcpyDeviceToDevice, s));
  }
  return IFK_OK;
}

}  // namespace

extern "C" {

int ifk_finalize_batched(int nfactors, const float* const* R_in, const int64_t* ldR,
                         const int64_t* rows_R, const int64_t* n, const double* rows_total,
                         double damping, void* const* R_out, const int64_t* ld_out, int out_dtype,
                         int prec, int* d_status, void* workspace, size_t workspace_bytes,
                         ifk_stream_t stream) {
  return finalize_many(nfactors, R_in, ldR, rows_R, n, rows_total, damping, R_out, ld_out, out_dtype, prec, d_status,
                       nullptr, workspace, workspace_bytes, stream);
}

int ifk_finalize_many(int nfactors, const float* const* R_in, const int64_t* ldR, const int64_t* rows_R,
                      const int64_t* n, const double* rows_total, double damping, void* const* R_out,
                      const int64_t* ld_out, int out_dtype, int prec, int* const* d_status, void* workspace,
                      size_t workspace_bytes, ifk_stream_t stream) {
  return finalize_many(nfactors, R_in, ldR, rows_R, n, rows_total, damping, R_out, ld_out, out_dtype, prec,
                       nullptr, d_status, workspace, workspace_bytes, stream);
}

// Workspace of the persistent bf16 solves: inverses of R_G | inverses of R_X |
// scratch of the larger solve (the left solves are n_out x n_out against n_in
// right-hand sides, the right ones the reverse).
size_t ifk_natgrad_workspace(int64_t n_out, int64_t n_in) {
  if (n_out <= 0 || n_in <= 0) return 0;
  size_t b = std::max(std::max(trsm_tc_workspace(n_out), trsm_tc_workspace(n_in)), natgrad_persist_bytes(n_out, n_in));
  if (needs_pad(n_out, n_in)) b = std::max(b, padded_natgrad_bytes(n_out, n_in));
  return align_up(b);
}

// The solves of ifk_natgrad (both = true: R_G^-1 R_G^-T g R_X^-1 R_X^-T) or of
// ifk_posterior_sample (both = false: R_G^-1 g R_X^-T, the transposed stages left out).
static int kron_solves(const float* grad_W, int64_t ld_g, const void* R_X, int64_t ld_rx, const void* R_G,
                       int64_t ld_rg, int r_dtype, float* nat, int64_t ld_nat, int64_t n_out, int64_t n_in,
                       int prec, int* d_status, void* workspace, size_t workspace_bytes, ifk_stream_t stream,
                       bool both) {
  if (!grad_W || !R_X || !R_G || !nat) return IFK_ERR_ARG;
  if (n_out <= 0 || n_in <= 0 || ld_g < n_in || ld_nat < n_in || ld_rx < n_in || ld_rg < n_out)
    return IFK_ERR_SHAPE;
  if (!dtype_ok(r_dtype)) return IFK_ERR_DTYPE;
  if (!prec_ok(prec)) return IFK_ERR_ARG;
  if (prec == IFK_PREC_AUTO) prec = r_dtype == IFK_BF16 ? IFK_PREC_BF16 : IFK_PREC_FP32;
  if (prec == IFK_PREC_BF16 &&
      (!workspace || !aligned(workspace) || workspace_bytes < ifk_natgrad_workspace(n_out, n_in)))
    return IFK_ERR_WORKSPACE;
  cudaStream_t s = S(stream);
  int rc;
  if (prec == IFK_PREC_BF16 && r_dtype == IFK_BF16 && needs_pad(n_out, n_in)) {
    // the persistent solves on the padded problem, then the leading block back
    Padded P;
    rc = pad_problem((uint8_t*)workspace, R_G, ld_rg, R_X, ld_rx, grad_W, ld_g, nullptr, n_out, n_in, P, s);
    if (rc != IFK_OK) return rc;
    rc = trsm_persist_prepare(P.Rg, P.po, P.po, P.inv_g, P.Rx, P.pi, P.pi, P.inv_x, s);
    if (rc != IFK_OK) return rc;
    if (both) rc = trsm_persist_run(P.Rg, P.po, 1, P.B, P.pi, 1, P.po, P.pi, P.inv_g, P.scratch, d_status, s);
    if (rc != IFK_OK) return rc;
    rc = trsm_persist_run(P.Rg, P.po, 0, P.B, P.pi, 1, P.po, P.pi, P.inv_g, P.scratch, d_status, s);
    if (rc != IFK_OK) return rc;
    if (both) rc = trsm_persist_run(P.Rx, P.pi, 1, P.B, 1, P.pi, P.pi, P.po, P.inv_x, P.scratch, d_status, s);
    if (rc != IFK_OK) return rc;
    rc = trsm_persist_run(P.Rx, P.pi, 0, P.B, 1, P.pi, P.pi, P.po, P.inv_x, P.scratch, d_status, s);
    if (rc != IFK_OK) return rc;
    IFK_CUDA_TRY(cudaMemcpy2DAsync(nat, ld_nat * sizeof(float), P.B, P.pi * sizeof(float), n_in * sizeof(float),
                                   n_out, cudaMemcpyDeviceToDevice, s));
    return IFK_OK;
  }
  if (nat != grad_W || ld_nat != ld_g) {
    IFK_CUDA_TRY(cudaMemcpy2DAsync(nat, ld_nat * sizeof(float), grad_W, ld_g * sizeof(float),
                                   n_in * sizeof(float), n_out, cudaMemcpyDeviceToDevice, s));
  }
  if (prec == IFK_PREC_BF16 && r_dtype == IFK_BF16 && trsm_persist_ok(R_G, ld_rg, n_out) &&
      trsm_persist_ok(R_X, ld_rx, n_in)) {
    // persistent tensor-core solves; the diagonal-block inverses of both factors in one launch
    const __nv_bfloat16* rg = (const __nv_bfloat16*)R_G;
    const __nv_bfloat16* rx = (const __nv_bfloat16*)R_X;
    uint8_t* inv_g = (uint8_t*)workspace;
    uint8_t* inv_x = inv_g + align_up(trsm_persist_inverse_bytes(n_out));
    uint8_t* scratch = inv_x + align_up(trsm_persist_inverse_bytes(n_in));
    rc = trsm_persist_prepare(rg, ld_rg, n_out, inv_g, rx, ld_rx, n_in, inv_x, s);
    if (rc != IFK_OK) return rc;
    if (both) rc = trsm_persist_run(rg, ld_rg, 1, nat, ld_nat, 1, n_out, n_in, inv_g, scratch, d_status, s);
    if (rc != IFK_OK) return rc;
    rc = trsm_persist_run(rg, ld_rg, 0, nat, ld_nat, 1, n_out, n_in, inv_g, scratch, d_status, s);
    if (rc != IFK_OK) return rc;
    if (both) rc = trsm_persist_run(rx, ld_rx, 1, nat, 1, ld_nat, n_in, n_out, inv_x, scratch, d_status, s);
    if (rc != IFK_OK) return rc;
    return trsm_persist_run(rx, ld_rx, 0, nat, 1, ld_nat, n_in, n_out, inv_x, scratch, d_status, s);
  }
  // left: R_G^T T1 = g ; R_G T2 = T1   (columns of nat are independent right-hand sides)
  rc = both ? trsm_run(R_G, ld_rg, r_dtype, 1, nat, ld_nat, 1, n_out, n_in, prec, workspace, d_status, s) : IFK_OK;
  if (rc != IFK_OK) return rc;
  rc = trsm_run(R_G, ld_rg, r_dtype, 0, nat, ld_nat, 1, n_out, n_in, prec, workspace, d_status, s);
  if (rc != IFK_OK) return rc;
  // right: R_X^T T3^T = T2^T ; R_X T4^T = T3^T on the transposed view of nat
  rc = both ? trsm_run(R_X, ld_rx, r_dtype, 1, nat, 1, ld_nat, n_in, n_out, prec, workspace, d_status, s) : IFK_OK;
  if (rc != IFK_OK) return rc;
  return trsm_run(R_X, ld_rx, r_dtype, 0, nat, 1, ld_nat, n_in, n_out, prec, workspace, d_status, s);
}

int ifk_natgrad(const float* grad_W, int64_t ld_g, const void* R_X, int64_t ld_rx, const void* R_G,
                int64_t ld_rg, int r_dtype, float* nat, int64_t ld_nat, int64_t n_out, int64_t n_in,
                int prec, int* d_status, void* workspace, size_t workspace_bytes,
                ifk_stream_t stream) {
  return kron_solves(grad_W, ld_g, R_X, ld_rx, R_G, ld_rg, r_dtype, nat, ld_nat, n_out, n_in, prec, d_status,
                     workspace, workspace_bytes, stream, true);
}

size_t ifk_natgrad_update_workspace(int64_t n_out, int64_t n_in) {
  if (n_out <= 0 || n_in <= 0) return 0;
  return ifk_natgrad_workspace(n_out, n_in) + align_up((size_t)n_out * n_in * sizeof(float)) +
         ifk_update_workspace(n_out * n_in);
}

int ifk_natgrad_update(const float* grad_W, int64_t ld_g, const void* R_X, int64_t ld_rx, const void* R_G,
                       int64_t ld_rg, int r_dtype, float* W, float* buf, int64_t n_out, int64_t n_in, double lr,
                       double momentum, double weight_decay, int buf_is_new, int prec, int* d_status,
                       void* workspace, size_t workspace_bytes, ifk_stream_t stream) {
  if (!grad_W || !R_X || !R_G || !W || (momentum > 0 && !buf)) return IFK_ERR_ARG;
  if (n_out <= 0 || n_in <= 0 || ld_g < n_in || ld_rx < n_in || ld_rg < n_out) return IFK_ERR_SHAPE;
  if (!dtype_ok(r_dtype)) return IFK_ERR_DTYPE;
  if (!prec_ok(prec)) return IFK_ERR_ARG;
  if (!workspace || !aligned(workspace) || workspace_bytes < ifk_natgrad_update_workspace(n_out, n_in))
    return IFK_ERR_WORKSPACE;
  if (prec == IFK_PREC_AUTO) prec = r_dtype == IFK_BF16 ? IFK_PREC_BF16 : IFK_PREC_FP32;
  cudaStream_t s = S(stream);
  uint8_t* ws = (uint8_t*)workspace;
  const size_t ngw = ifk_natgrad_workspace(n_out, n_in);
  float* nat = (float*)(ws + ngw);
  void* uws = ws + ngw + align_up((size_t)n_out * n_in * sizeof(float));
  // The natural gradient into the workspace, then one update pass.  Applying the
  // update in the last solve's epilogue instead (W and buf read and written there, no
  // natural gradient stored) was built and measured: at n = 4096 it was 0.28 ms
  // slower than this sequence, since the epilogue warps are on the solve's critical
  // path and the separate pass runs on every SM at HBM speed.
  int rc = ifk_natgrad(grad_W, ld_g, R_X, ld_rx, R_G, ld_rg, r_dtype, nat, n_in, n_out, n_in, prec, d_status,
                       workspace, ngw, stream);
  if (rc != IFK_OK) return rc;
  return update_run(W, buf, nat, n_out * n_in, lr, momentum, weight_decay, 0.0, buf_is_new, (double*)uws, s);
}

size_t ifk_posterior_sample_workspace(int64_t n_out, int64_t n_in) { return ifk_natgrad_workspace(n_out, n_in); }

int ifk_posterior_sample(const float* xi, int64_t ld_xi, const void* C_A, int64_t ld_ca, const void* C_G,
                         int64_t ld_cg, int c_dtype, float* out, int64_t ld_out, int64_t n_out, int64_t n_in,
                         int prec, int* d_status, void* workspace, size_t workspace_bytes,
                         ifk_stream_t stream) {
  return kron_solves(xi, ld_xi, C_A, ld_ca, C_G, ld_cg, c_dtype, out, ld_out, n_out, n_in, prec, d_status,
                     workspace, workspace_bytes, stream, false);
}

// a layer's slice of the batched workspace: ifk_natgrad's | the bias solves' scratch
static size_t natgrad_batched_slice(int64_t n_out, int64_t n_in) {
  return ifk_natgrad_workspace(n_out, n_in) +
         align_up(std::max(trsm_persist_workspace(n_out, 1), trsm_persist_workspace(pad8(n_out), 1)));
}

size_t ifk_natgrad_batched_workspace(int nlayers, const int64_t* n_out, const int64_t* n_in) {
  if (nlayers <= 0 || !n_out || !n_in) return 0;
  size_t b = 0;
  for (int l = 0; l < nlayers; ++l) {
    if (n_out[l] <= 0 || n_in[l] <= 0) return 0;
    b += natgrad_batched_slice(n_out[l], n_in[l]);
  }
  return b;
}

int ifk_natgrad_batched(int nlayers, const float* const* grad_W, const int64_t* ld_g, const void* const* R_X,
                        const int64_t* ld_rx, const void* const* R_G, const int64_t* ld_rg, int r_dtype,
                        float* const* nat, const int64_t* ld_nat, const int64_t* n_out, const int64_t* n_in,
                        const float* const* grad_b, float* const* nat_b, int prec, int* d_status, void* workspace,
                        size_t workspace_bytes, ifk_stream_t stream) {
  if (nlayers < 0 || (nlayers > 0 && (!grad_W || !ld_g || !R_X || !ld_rx || !R_G || !ld_rg || !nat || !ld_nat ||
                                      !n_out || !n_in)))
    return IFK_ERR_ARG;
  if ((grad_b == nullptr) != (nat_b == nullptr)) return IFK_ERR_ARG;
  auto has_bias = [&](int l) { return grad_b && grad_b[l]; };
  for (int l = 0; l < nlayers; ++l)
    if (grad_b && (grad_b[l] == nullptr) != (nat_b[l] == nullptr)) return IFK_ERR_ARG;
  if (!dtype_ok(r_dtype)) return IFK_ERR_DTYPE;
  if (!prec_ok(prec)) return IFK_ERR_ARG;
  for (int l = 0; l < nlayers; ++l) {
    if (!grad_W[l] || !R_X[l] || !R_G[l] || !nat[l]) return IFK_ERR_ARG;
    if (n_out[l] <= 0 || n_in[l] <= 0 || ld_g[l] < n_in[l] || ld_nat[l] < n_in[l] || ld_rx[l] < n_in[l] ||
        ld_rg[l] < n_out[l])
      return IFK_ERR_SHAPE;
  }
  if (nlayers == 0) return IFK_OK;
  if (!workspace || !aligned(workspace) ||
      workspace_bytes < ifk_natgrad_batched_workspace(nlayers, n_out, n_in))
    return IFK_ERR_WORKSPACE;
  if (prec == IFK_PREC_AUTO) prec = r_dtype == IFK_BF16 ? IFK_PREC_BF16 : IFK_PREC_FP32;
  cudaStream_t s = S(stream);
  // each layer owns the slice of the workspace ifk_natgrad would take, then its bias scratch
  std::vector<char*> wsl((size_t)nlayers);
  {
    char* w = (char*)workspace;
    for (int l = 0; l < nlayers; ++l) {
      wsl[l] = w;
      w += natgrad_batched_slice(n_out[l], n_in[l]);
    }
  }
  // the layers of the persistent bf16 path share launches; the others go one by one
  // (orders that are not multiples of 8 join them on their padded problem, as ifk_natgrad does)
  std::vector<int> batch;
  const bool bf = prec == IFK_PREC_BF16 && r_dtype == IFK_BF16;
  for (int l = 0; l < nlayers; ++l) {
    const bool pers = bf && (needs_pad(n_out[l], n_in[l]) ||
                             (trsm_persist_ok(R_G[l], ld_rg[l], n_out[l]) && trsm_persist_ok(R_X[l], ld_rx[l], n_in[l])));
    if (pers) {
      batch.push_back(l);
      continue;
    }
    int rc = ifk_natgrad(grad_W[l], ld_g[l], R_X[l], ld_rx[l], R_G[l], ld_rg[l], r_dtype, nat[l], ld_nat[l],
                         n_out[l], n_in[l], prec, d_status, wsl[l], ifk_natgrad_workspace(n_out[l], n_in[l]),
                         stream);
    if (rc != IFK_OK) return rc;
    if (has_bias(l)) {
      rc = ifk_natgrad_bias(grad_b[l], R_G[l], ld_rg[l], r_dtype, nat_b[l], n_out[l], prec, nullptr, 0, stream);
      if (rc != IFK_OK) return rc;
    }
  }
  const int nb = (int)batch.size();
  if (nb == 0) return IFK_OK;
  // layout of a layer's slice: inverses of R_G | inverses of R_X | solve scratch (as ifk_natgrad)
  std::vector<const __nv_bfloat16*> A((size_t)2 * nb);
  std::vector<int64_t> ld((size_t)2 * nb), nn((size_t)2 * nb);
  std::vector<void*> inv((size_t)2 * nb);
  std::vector<TrsmProblem> pg((size_t)nb), px((size_t)nb), pl;
  std::vector<std::pair<int, Padded>> padded;
  for (int i = 0; i < nb; ++i) {
    const int l = batch[i];
    if (needs_pad(n_out[l], n_in[l])) {
      Padded P;
      int rc = pad_problem((uint8_t*)wsl[l], R_G[l], ld_rg[l], R_X[l], ld_rx[l], grad_W[l], ld_g[l],
                           has_bias(l) ? grad_b[l] : nullptr, n_out[l], n_in[l], P, s);
      if (rc != IFK_OK) return rc;
      A[2 * i] = P.Rg;
      ld[2 * i] = P.po;
      nn[2 * i] = P.po;
      inv[2 * i] = P.inv_g;
      A[2 * i + 1] = P.Rx;
      ld[2 * i + 1] = P.pi;
      nn[2 * i + 1] = P.pi;
      inv[2 * i + 1] = P.inv_x;
      pg[i] = TrsmProblem{P.Rg, P.po, P.B, P.pi, 1, P.po, P.pi, P.inv_g, P.scratch};
      px[i] = TrsmProblem{P.Rx, P.pi, P.B, 1, P.pi, P.pi, P.po, P.inv_x, P.scratch};
      if (has_bias(l))
        pl.push_back(TrsmProblem{P.Rg, P.po, P.b, 1, 1, P.po, 1, P.inv_g,
                                 wsl[l] + ifk_natgrad_workspace(n_out[l], n_in[l])});
      padded.emplace_back(l, P);
      continue;
    }
    if (nat[l] != grad_W[l] || ld_nat[l] != ld_g[l])
      IFK_CUDA_TRY(cudaMemcpy2DAsync(nat[l], ld_nat[l] * sizeof(float), grad_W[l], ld_g[l] * sizeof(float),
                                     n_in[l] * sizeof(float), n_out[l], cudaMemcpyDeviceToDevice, s));
    uint8_t* inv_g = (uint8_t*)wsl[l];
    uint8_t* inv_x = inv_g + align_up(trsm_persist_inverse_bytes(n_out[l]));
    uint8_t* scratch = inv_x + align_up(trsm_persist_inverse_bytes(n_in[l]));
    A[2 * i] = (const __nv_bfloat16*)R_G[l];
    ld[2 * i] = ld_rg[l];
    nn[2 * i] = n_out[l];
    inv[2 * i] = inv_g;
    A[2 * i + 1] = (const __nv_bfloat16*)R_X[l];
    ld[2 * i + 1] = ld_rx[l];
    nn[2 * i + 1] = n_in[l];
    inv[2 * i + 1] = inv_x;
    // left solves on the columns of nat, right solves on its transposed view
    pg[i] = TrsmProblem{(const __nv_bfloat16*)R_G[l], ld_rg[l], nat[l], ld_nat[l], 1, n_out[l], n_in[l], inv_g, scratch};
    px[i] = TrsmProblem{(const __nv_bfloat16*)R_X[l], ld_rx[l], nat[l], 1, ld_nat[l], n_in[l], n_out[l], inv_x, scratch};
    if (has_bias(l)) {
      // the bias: one more right-hand side of the left solves (R_G^-1 R_G^-T g_b), own scratch
      if (nat_b[l] != grad_b[l])
        IFK_CUDA_TRY(cudaMemcpyAsync(nat_b[l], grad_b[l], n_out[l] * sizeof(float), cudaMemcpyDeviceToDevice, s));
      pl.push_back(TrsmProblem{(const __nv_bfloat16*)R_G[l], ld_rg[l], nat_b[l], 1, 1, n_out[l], 1, inv_g,
                               wsl[l] + ifk_natgrad_workspace(n_out[l], n_in[l])});
    }
  }
  std::vector<TrsmProblem> left(pg);
  left.insert(left.end(), pl.begin(), pl.end());
  int rc = trsm_persist_prepare_many(2 * nb, A.data(), ld.data(), nn.data(), inv.data(), s);
  if (rc != IFK_OK) return rc;
  // R_G^T T1 = g; R_G T2 = T1; R_X^T T3^T = T2^T; R_X T4^T = T3^T, each stage for every layer at once
  rc = trsm_persist_run_many((int)left.size(), left.data(), 1, d_status, s);
  if (rc != IFK_OK) return rc;
  rc = trsm_persist_run_many((int)left.size(), left.data(), 0, d_status, s);
  if (rc != IFK_OK) return rc;
  rc = trsm_persist_run_many(nb, px.data(), 1, d_status, s);
  if (rc != IFK_OK) return rc;
  rc = trsm_persist_run_many(nb, px.data(), 0, d_status, s);
  if (rc != IFK_OK) return rc;
  for (const auto& e : padded) {  // the leading blocks of the padded problems
    const int l = e.first;
    const Padded& P = e.second;
    IFK_CUDA_TRY(cudaMemcpy2DAsync(nat[l], ld_nat[l] * sizeof(float), P.B, P.pi * sizeof(float),
                                   n_in[l] * sizeof(float), n_out[l], cudaMemcpyDeviceToDevice, s));
    if (has_bias(l))
      IFK_CUDA_TRY(cudaMemcpyAsync(nat_b[l], P.b, n_out[l] * sizeof(float), cudaMemcpyDeviceToDevice, s));
  }
  return IFK_OK;
}

int ifk_natgrad_bias(const float* grad_b, const void* R_G, int64_t ld_rg, int r_dtype, float* nat_b,
                     int64_t n_out, int prec, void* workspace, size_t workspace_bytes,
                     ifk_stream_t stream) {
  (void)workspace;
  (void)workspace_bytes;
  if (!grad_b || !R_G || !nat_b) return IFK_ERR_ARG;
  if (n_out <= 0 || ld_rg < n_out) return IFK_ERR_SHAPE;
  if (!dtype_ok(r_dtype)) return IFK_ERR_DTYPE;
  if (!prec_ok(prec)) return IFK_ERR_ARG;
  cudaStream_t s = S(stream);
  if (nat_b != grad_b)
    IFK_CUDA_TRY(cudaMemcpyAsync(nat_b, grad_b, n_out * sizeof(float), cudaMemcpyDeviceToDevice, s));
  // a single right-hand side: the fp32 path (tensor-core tiles would be 1/64 full)
  int rc = trsm_run(R_G, ld_rg, r_dtype, 1, nat_b, 1, 1, n_out, 1, IFK_PREC_FP32, nullptr, nullptr, s);
  if (rc != IFK_OK) return rc;
  return trsm_run(R_G, ld_rg, r_dtype, 0, nat_b, 1, 1, n_out, 1, IFK_PREC_FP32, nullptr, nullptr, s);
}

size_t ifk_update_workspace(int64_t count) {
  (void)count;
  return ALIGN;
}

int ifk_update(float* W, float* buf, const float* nat, int64_t count, double lr, double momentum,
               double weight_decay, double grad_clip, int buf_is_new, void* workspace,
               size_t workspace_bytes, ifk_stream_t stream) {
  if (!W || !nat || (momentum > 0 && !buf)) return IFK_ERR_ARG;
  if (count < 0) return IFK_ERR_SHAPE;
  if (grad_clip > 0 && (!workspace || !aligned(workspace) || workspace_bytes < sizeof(double)))
    return IFK_ERR_WORKSPACE;
  return update_run(W, buf, nat, count, lr, momentum, weight_decay, grad_clip, buf_is_new,
                    (double*)workspace, S(stream));
}

int ifk_update_bias(float* b, const float* nat_b, int64_t count, double lr, double weight_decay,
                    ifk_stream_t stream) {
  if (!b || !nat_b) return IFK_ERR_ARG;
  if (count < 0) return IFK_ERR_SHAPE;
  return update_bias_run(b, nat_b, count, lr, weight_decay, S(stream));
}

}  // extern "C"
