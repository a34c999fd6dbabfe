"""Forward/backward hooks that stream captured activations into device R factors.

Mirror of the reference's ``RawActivationHooks`` (ifkfac/activation_hooks.py):
same constructor, same lifecycle (enable / get_factors / clear / remove /
flush / pause / resume / capture / n_samples_accumulated), same chunk
preprocessing (3-D reshape with random row subsampling, Conv2d im2col with
subsampling, optional ones column, optional chunk transforms) and the same
three accumulation modes (streaming, batched flush, deferred window).  The
folds, the damping fold and the checks run in libifk.so: each factor keeps an
n x n fp32 buffer on the device plus the host row counts, and
``_R_X[module]`` / ``_R_G[module]`` are views of the reference's trapezoidal
running R (``R[:min(rows, n)]``).  Chunks may be bf16 (autocast): they are
folded natively on the tensor cores, where the reference's geqrf has no bf16
kernel.
"""
from __future__ import annotations

import logging
import warnings
from contextlib import contextmanager
from typing import Dict, List, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib
from .engine import Factor, Rows, as_rows, fold_segments

logger = logging.getLogger(__name__)

warnings.filterwarnings("ignore", message="Full backward hook is firing", category=UserWarning)


class IFKFACRankError(RuntimeError):
    """Raised when accumulated p < n for a layer, making QR rank-deficient."""


def unfold_conv_input(x: torch.Tensor, module: nn.Conv2d) -> torch.Tensor:
    """im2col rows (B*L, C_in*kH*kW) (ifkfac/activation_hooks.py:489-499)."""
    x_unf = F.unfold(x, kernel_size=module.kernel_size, dilation=module.dilation,
                     padding=module.padding, stride=module.stride)
    B, C_kk, L = x_unf.shape
    return x_unf.permute(0, 2, 1).reshape(B * L, C_kk)


def reshape_conv_grad(delta: torch.Tensor) -> torch.Tensor:
    """(B*H_out*W_out, C_out) rows (ifkfac/activation_hooks.py:501-504)."""
    B, C_out, H, W = delta.shape
    return delta.permute(0, 2, 3, 1).reshape(B * H * W, C_out)


def prepare_x(x: torch.Tensor, module: nn.Module, max_conv_rows: int, max_seq_rows: int,
              augment_bias: bool, transform=None):
    """Activation rows of one forward call (ifkfac/activation_hooks.py:519-548).

    The rows are returned as :class:`Rows`: the 3-D reshape is a view; the
    random row subsample, the bias column and a Conv2d input's im2col rows are
    read in place by the fold kernels instead of being copied.  With a chunk transform the rows are
    materialised and the transform's output (a tensor) is returned."""
    idx = None
    if isinstance(module, nn.Conv2d):
        # im2col rows read in place by the fold (no F.unfold copy); the same rows and
        # the same random subsample as the reference's unfold + randperm
        rows = Rows.conv2d(x, module)
        if max_conv_rows > 0 and rows.rows > max_conv_rows:
            rows = Rows.conv2d(x, module, torch.randperm(rows.rows, device=x.device)[:max_conv_rows])
        if transform is not None:
            return transform(rows.materialize())
        return rows
    elif x.ndim > 2:
        x = x.reshape(-1, x.shape[-1])
        if max_seq_rows > 0 and x.shape[0] > max_seq_rows:
            idx = torch.randperm(x.shape[0], device=x.device)[:max_seq_rows]
    ones = augment_bias and isinstance(module, nn.Linear) and module.bias is not None
    rows = Rows(x, idx, ones)
    if transform is not None:
        return transform(rows.materialize())
    return rows


def prepare_g(delta: torch.Tensor, module: nn.Module, max_seq_rows: int, transform=None):
    """Gradient rows of one backward call (ifkfac/activation_hooks.py:601-615), as
    :class:`Rows` (or the transform's output)."""
    idx = None
    if isinstance(module, nn.Conv2d):
        delta = reshape_conv_grad(delta)
    elif delta.ndim > 2:
        delta = delta.reshape(-1, delta.shape[-1])
        if max_seq_rows > 0 and delta.shape[0] > max_seq_rows:
            idx = torch.randperm(delta.shape[0], device=delta.device)[:max_seq_rows]
    rows = Rows(delta, idx)
    if transform is not None:
        return transform(rows.materialize())
    return rows


def _rows_count(c) -> int:
    return c.rows if isinstance(c, Rows) else int(c.shape[0])


class RawActivationHooks:
    """Forward/backward hooks that maintain streaming-TSQR R factors on the device.

    Parameters are those of the reference (ifkfac/activation_hooks.py:128-216);
    ``precision`` selects the fold arithmetic (``_lib.PREC_AUTO``: tensor cores
    for bf16 chunks, fp32 CUDA cores for fp32 chunks).
    """

    _SEQ_SUBSAMPLE: int = 2048

    def __init__(self, model: nn.Module, damping: float = 1e-2, max_out_dim: int = 0,
                 augment_bias: bool = False, max_conv_rows: int = 512,
                 max_seq_rows: Optional[int] = None, batched: bool = False, deferred: bool = False,
                 deferred_window: int = 5, precision: int = _lib.PREC_AUTO):
        if batched and deferred:
            raise ValueError("batched and deferred modes are mutually exclusive")
        self.model = model
        self.damping = damping
        self.augment_bias = augment_bias
        self.max_conv_rows = max_conv_rows
        self.max_seq_rows = self._SEQ_SUBSAMPLE if max_seq_rows is None else max_seq_rows
        self.batched = batched
        self.deferred = deferred
        self.deferred_window = deferred_window
        self.precision = precision
        self.chunk_transform_X = None
        self.chunk_transform_G = None
        self._handles: List = []
        self._enabled = False
        self._fx: Dict[nn.Module, Optional[Factor]] = {}
        self._fg: Dict[nn.Module, Optional[Factor]] = {}
        self._n_rows_X: Dict[nn.Module, int] = {}
        self._n_rows_G: Dict[nn.Module, int] = {}
        self._pending_X: Dict[nn.Module, List[torch.Tensor]] = {}
        self._pending_G: Dict[nn.Module, List[torch.Tensor]] = {}
        self._raw_X: Dict[nn.Module, List[torch.Tensor]] = {}
        self._raw_G: Dict[nn.Module, List[torch.Tensor]] = {}
        self._ws: Dict[Tuple, torch.Tensor] = {}
        self._linear_layers: List[nn.Module] = []
        for module in model.modules():
            if not isinstance(module, (nn.Linear, nn.Conv2d)):
                continue
            if max_out_dim > 0:
                out_dim = module.out_features if isinstance(module, nn.Linear) else module.out_channels
                if out_dim > max_out_dim:
                    continue
            self._linear_layers.append(module)
            self._fx[module] = None
            self._fg[module] = None
            self._n_rows_X[module] = 0
            self._n_rows_G[module] = 0
            self._pending_X[module] = []
            self._pending_G[module] = []
            self._raw_X[module] = []
            self._raw_G[module] = []

    # ---- estimator interface ----
    @property
    def linear_layers(self) -> List[nn.Module]:
        return self._linear_layers

    @property
    def is_enabled(self) -> bool:
        return self._enabled

    @property
    def _R_X(self) -> Dict[nn.Module, Optional[torch.Tensor]]:
        """Running R_X per layer in the reference's shape (min(rows, n), n), or None."""
        return {m: (None if f is None or f.rows_seen == 0 else f.R[: f.rows_R]) for m, f in self._fx.items()}

    @property
    def _R_G(self) -> Dict[nn.Module, Optional[torch.Tensor]]:
        return {m: (None if f is None or f.rows_seen == 0 else f.R[: f.rows_R]) for m, f in self._fg.items()}

    def enable(self) -> None:
        if self._enabled:
            return
        for module in self._linear_layers:
            self._handles.append(module.register_forward_hook(self._forward_hook))
            self._handles.append(module.register_full_backward_hook(self._backward_hook))
        self._enabled = True

    def pause(self) -> None:
        self._enabled = False

    def resume(self) -> None:
        self._enabled = True

    @contextmanager
    def capture(self):
        previous = getattr(self, "_enabled", False)
        self._enabled = True
        try:
            yield self
        finally:
            self._enabled = previous

    def n_samples_accumulated(self, module: Optional[nn.Module] = None) -> int:
        target = module or (self._linear_layers[0] if self._linear_layers else None)
        return 0 if target is None else self._n_rows_X.get(target, 0)

    # ---- device state ----
    def _factor(self, table, module, n: int, device) -> Factor:
        f = table[module]
        if f is None or f.n != n:
            f = Factor(n, device, self.precision)
            table[module] = f
        return f

    def _workspace(self, key, nbytes, device) -> torch.Tensor:
        ws = self._ws.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)
            self._ws[key] = ws
        return ws

    def _fold_lists(self, table, items) -> None:
        """Fold (module, [chunks]) pairs of one table (see _fold_entries)."""
        self._fold_entries([(table, m, chunks) for m, chunks in items])

    def _fold_entries(self, entries) -> None:
        """Fold (table, module, [chunks]) entries: every module's chunks in arrival
        order, all of them in one ifk_tsqr_fold_segments call per device (no
        concatenation; the bucketed flush of ifkfac/activation_hooks.py:370-457 and
        the deferred drain of :347-364).  With an explicit precision the chunks may
        mix fp32 and bf16 (each segment carries its type); with PREC_AUTO the
        precision follows the chunk type, so the dtypes fold in separate calls."""
        groups: Dict[Tuple, List] = {}
        for table, module, chunks in entries:
            rs = [as_rows(c) for c in chunks]
            rs = [r for r in rs if r.rows > 0]
            if not rs:
                continue
            if not rs[0].x.is_cuda:
                raise ValueError("ifkfac_b200 hooks need CUDA activations (no CPU path)")
            key = (rs[0].device, None if self.precision != _lib.PREC_AUTO else rs[0].dtype)
            groups.setdefault(key, []).append((table, module, rs))
        for (dev, dt), lst in groups.items():
            fs = [self._factor(table, m, rs[0].cols, dev) for table, m, rs in lst]
            key = ("fold", dev)
            self._ws[key] = fold_segments(fs, [rs for _, _, rs in lst], self._ws.get(key))

    def _fold_now(self, table, module, chunk) -> None:
        self._fold_lists(table, [(module, [chunk])])

    # ---- hooks ----
    def _forward_hook(self, module, inp, out):
        if not self._enabled:
            return
        x = prepare_x(inp[0].detach(), module, self.max_conv_rows, self.max_seq_rows,
                      self.augment_bias, self.chunk_transform_X)
        self._accumulate(module, x, self._fx, self._n_rows_X, self._pending_X, self._raw_X)

    def _backward_hook(self, module, grad_input, grad_output):
        if not self._enabled:
            return
        d = prepare_g(grad_output[0].detach(), module, self.max_seq_rows, self.chunk_transform_G)
        self._accumulate(module, d, self._fg, self._n_rows_G, self._pending_G, self._raw_G)

    def _accumulate(self, module, chunk, table, nrows, pending, raw):
        n = _rows_count(chunk)
        if self.deferred:
            raw[module].append(chunk)
            nrows[module] += n
            if len(raw[module]) >= self.deferred_window:
                self._fold_lists(table, [(module, raw[module])])
                raw[module] = []
            return
        if self.batched:
            pending[module].append(chunk)
            nrows[module] += n
            return
        self._fold_now(table, module, chunk)
        nrows[module] += n

    def flush(self) -> None:
        """Batched mode: fold every pending chunk (no-op otherwise)."""
        if not self.batched:
            return
        self._fold_pending(((self._pending_X, self._fx), (self._pending_G, self._fg)))

    def _drain_deferred(self) -> None:
        self._fold_pending(((self._raw_X, self._fx), (self._raw_G, self._fg)))

    def _fold_pending(self, sources) -> None:
        """X and delta chunks of every layer in one call (they share launches)."""
        entries = []
        for pending, table in sources:
            for m, chunks in pending.items():
                if chunks:
                    entries.append((table, m, chunks))
                    pending[m] = []
        if entries:
            self._fold_entries(entries)

    # ---- factors ----
    def get_factors(self, out_dtype: torch.dtype = torch.float32,
                    status: Optional[torch.Tensor] = None) -> Dict[nn.Module, Tuple[torch.Tensor, torch.Tensor]]:
        """Damped R factors per layer with data: finalize_R(R / sqrt(rows), damping)
        (ifkfac/activation_hooks.py:240-341).  Layers whose R is still trapezoidal
        are skipped; in batched mode they raise IFKFACRankError, as in the reference."""
        if self.deferred:
            self._drain_deferred()
        factors = {}
        L = _lib.lib()
        self.last_status = None
        self.status_index = {}
        ready = []
        for module in self._linear_layers:
            fx, fg = self._fx[module], self._fg[module]
            if fx is None or fg is None or fx.rows_seen == 0 or fg.rows_seen == 0:
                continue
            if fx.rows_R < fx.n or fg.rows_R < fg.n:
                continue
            rows_X, rows_G = self._n_rows_X[module], self._n_rows_G[module]
            if self.batched:
                if rows_X < fx.n:
                    raise IFKFACRankError(f"Layer {module}: accumulated {rows_X} rows for X, "
                                          f"but need >= n_in={fx.n} (batched mode).")
                if rows_G < fg.n:
                    raise IFKFACRankError(f"Layer {module}: accumulated {rows_G} rows for δ, "
                                          f"but need >= n_out={fg.n} (batched mode).")
            ready.append((module, fx, fg, rows_X, rows_G))
        if not ready:
            return factors
        import ctypes
        arr = lambda t, v: (t * len(v))(*v)
        dev = ready[0][1].R.device
        # one device status word per layer: the fused finite check of the damping fold
        self.last_status = torch.zeros(len(self._linear_layers), dtype=torch.int32, device=dev)
        # the layers of one precision finalize together (ifk_finalize_batched: the
        # damping folds of up to 16 factors share a launch)
        groups = {}
        for module, fx, fg, rows_X, rows_G in ready:
            prec = _lib.PREC_BF16 if (out_dtype == torch.bfloat16 or fx.prec == _lib.PREC_BF16) else self.precision
            groups.setdefault((prec, fx.R.device), []).append((module, fx, fg, rows_X, rows_G))
        for (prec, dev), lst in groups.items():
            fs, outs, rows, sts = [], [], [], []
            for module, fx, fg, rows_X, rows_G in lst:
                self.status_index[module] = len(self.status_index)
                pair = [torch.empty(f.n, f.n, dtype=out_dtype, device=dev) for f in (fx, fg)]
                factors[module] = (pair[0], pair[1])
                fs += [fx, fg]
                outs += pair
                rows += [float(rows_X), float(rows_G)]
            ns = [f.n for f in fs]
            ws = self._workspace(("fin", dev), L.ifk_finalize_batched_workspace(len(fs), arr(ctypes.c_int64, ns)),
                                 dev)
            # one status word per layer (both of its factors write it): the caller's word
            # when given, else the layer's entry of last_status
            base = self.last_status.data_ptr()
            sts = []
            for module, *_ in lst:
                p = status.data_ptr() if status is not None else base + 4 * self.status_index[module]
                sts += [p, p]
            _lib.check(L.ifk_finalize_many(
                len(fs), arr(ctypes.c_void_p, [f.R.data_ptr() for f in fs]), arr(ctypes.c_int64, ns),
                arr(ctypes.c_int64, [f.rows_R for f in fs]), arr(ctypes.c_int64, ns),
                arr(ctypes.c_double, rows), float(self.damping),
                arr(ctypes.c_void_p, [o.data_ptr() for o in outs]), arr(ctypes.c_int64, ns),
                _lib.BF16 if out_dtype == torch.bfloat16 else _lib.F32, prec, arr(ctypes.c_void_p, sts),
                ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream), "ifk_finalize_many")
        return factors

    def clear(self) -> None:
        for module in self._linear_layers:
            for f in (self._fx[module], self._fg[module]):
                if f is not None:
                    f.clear()
            self._n_rows_X[module] = 0
            self._n_rows_G[module] = 0
            self._pending_X[module] = []
            self._pending_G[module] = []
            self._raw_X[module] = []
            self._raw_G[module] = []

    def remove(self) -> None:
        for h in self._handles:
            h.remove()
        self._handles.clear()
        self._enabled = False
        self.clear()
