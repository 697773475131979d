"""Bind the B200 segmented operators into a loaded DeepMD DPA4 model.

Same seam as the reference's ``python/model/fused_deepmd.py`` (lines
58-470): two DeepMD dispatch points are rebound, and every call keeps a
per-call fallback to DeepMD's own implementation.

``segment_envelope_gated_softmax`` (module attribute in DeepMD's
``sezm_nn.attention`` / ``sezm_nn.so2`` / ``sezm_nn``)
    replaced by ``ops.segment_softmax`` with the null logit
    ``log(softplus(z_bias) + eps)`` and the envelope folded into the logit.
``SO2Convolution.forward_envelope`` (per block instance)
    replaced by one ``ops.segment_sum`` with ``edge_scale = env * src_gate``
    and ``node_scale = inv_sqrt_deg``.
``edge_force_virial`` (module attribute, opt-in with ``force=True``)
    the per-atom force / virial scatter of DeepMD's post-processing, which the
    reference lists as not yet wired (``docs/deepmd-fused-dispatch.md:126``):
    ``(g, edge_vec, src, dst, n_ext) -> (force, atom_virial)`` replaced by
    ``ops.force_assembly`` with fp64 sums.

A call falls back -- counted in ``FusedStats`` and warned about once -- when a
precondition fails (training mode, a source-weighted softmax, non-contiguous
or non-fp32 or non-CUDA tensors, shape mismatch) or when the fused operator
raises.  The destination CSR view (offsets, stable order) is built on the
device (``destination_csr``: boundary kernel for sorted input, histogram and
stable device grouping otherwise) and kept in a small LRU keyed by the ``dst``
storage and version.
"""
from __future__ import annotations

import warnings
from dataclasses import dataclass, field
from types import MethodType
from typing import Any, Iterable

import torch
import torch.nn.functional as F

_CSR_CAPACITY = 4
# Host tests drive the seams with CPU tensors and a stand-in operator bundle;
# on a real install this guard keeps CPU tensors away from the CUDA kernels.
_ACCEPT_ANY_DEVICE = False
_SOFTMAX_NAME = "segment_envelope_gated_softmax"
_FORCE_NAME = "edge_force_virial"
_BLOCK_PREFIX = "block:"


@dataclass
class FusedStats:
    """Hit / fallback counters of the installed seams."""

    softmax_hits: int = 0
    softmax_fallbacks: int = 0
    envelope_hits: int = 0
    envelope_fallbacks: int = 0
    force_hits: int = 0
    force_fallbacks: int = 0
    bound_softmax: bool = False
    bound_envelope: bool = False
    bound_force: bool = False
    blocks: int = 0
    last_error: str | None = None

    def as_dict(self) -> dict[str, Any]:
        return {
            "softmax_hits": self.softmax_hits,
            "softmax_fallbacks": self.softmax_fallbacks,
            "envelope_hits": self.envelope_hits,
            "envelope_fallbacks": self.envelope_fallbacks,
            "force_hits": self.force_hits,
            "force_fallbacks": self.force_fallbacks,
            "bound_softmax": self.bound_softmax,
            "bound_envelope": self.bound_envelope,
            "bound_force": self.bound_force,
            "blocks": self.blocks,
            "last_error": self.last_error,
        }


def _usable_tensor(value: Any, *, dtype: torch.dtype = torch.float32) -> bool:
    if not isinstance(value, torch.Tensor):
        return False
    on_device = value.is_cuda or _ACCEPT_ANY_DEVICE
    return on_device and value.dtype == dtype and value.is_contiguous()


def _load_ops() -> Any:
    """The fused operator bundle, or ``None`` when it cannot run here."""
    try:
        from .. import kernels
    except ImportError:
        return None
    if not kernels.segment_available():
        return None
    return kernels


class _CsrView:
    """Destination CSR view ``(offsets, order)`` cached by the dst storage.

    With an operator bundle that has ``destination_csr`` (the B200 kernels)
    the view is built on the device: the boundary kernel for a
    destination-sorted list (``order`` is then ``None`` and the operators read
    the edges in place), the histogram + stable device grouping otherwise.
    Bundles without it fall back to their ``segment_offsets`` plus
    ``torch.argsort(dst, stable=True)`` as the reference does
    (``python/model/fused_deepmd.py:111-124``).  The cache key includes the
    tensor's version counter, so an in-place change of ``dst`` is not served
    a stale view.
    """

    def __init__(self, builder=None, capacity: int = _CSR_CAPACITY, csr=None) -> None:
        self._builder = builder
        self._csr = csr
        self._capacity = capacity
        self._cache: dict[tuple[int, ...], tuple[torch.Tensor, torch.Tensor | None]] = {}
        self._lru: list[tuple[int, ...]] = []

    def _offsets(self, dst: torch.Tensor, n_nodes: int) -> torch.Tensor:
        builder = self._builder
        if builder is None:
            from ..kernels.segment import segment_offsets as builder
        return builder(dst, n_nodes)

    def _build(self, dst: torch.Tensor, n_nodes: int):
        if self._csr is not None:
            return self._csr(dst, n_nodes)
        return self._offsets(dst, n_nodes), torch.argsort(dst, stable=True)

    def get(self, dst: torch.Tensor, n_nodes: int) -> tuple[torch.Tensor, torch.Tensor | None]:
        key = (int(dst.data_ptr()), int(dst.numel()), int(n_nodes), int(dst._version))
        hit = self._cache.get(key)
        if hit is not None:
            return hit
        view = self._build(dst, n_nodes)
        self._cache[key] = view
        self._lru.append(key)
        while len(self._lru) > self._capacity:
            self._cache.pop(self._lru.pop(0), None)
        return view


class _ForcePlan:
    """Destination-sorted copies of the index columns and the source grouping
    of one edge list, cached by the ``src`` / ``dst`` storages and versions.

    ``force_assembly`` walks destination segments in place, so an edge list
    that is not grouped by destination is permuted once (``dst_order``); the
    per-edge gradients are permuted with the same order on every call.
    """

    def __init__(self, csr: _CsrView, grouper=None, capacity: int = _CSR_CAPACITY) -> None:
        self._csr = csr
        self._grouper = grouper
        self._capacity = capacity
        self._cache: dict[tuple[int, ...], tuple] = {}
        self._lru: list[tuple[int, ...]] = []

    def get(self, src: torch.Tensor, dst: torch.Tensor, n_nodes: int):
        key = (int(src.data_ptr()), int(src._version), int(dst.data_ptr()), int(dst._version),
               int(dst.numel()), int(n_nodes))
        hit = self._cache.get(key)
        if hit is not None:
            return hit
        offsets, order = self._csr.get(dst, n_nodes)
        src_sorted = src if order is None else src.index_select(0, order)
        dst_sorted = dst if order is None else dst.index_select(0, order)
        grouper = self._grouper
        if grouper is None:
            from ..kernels.segment import group_by_source as grouper
        src_order, src_offsets = grouper(src_sorted.contiguous(), n_nodes)
        plan = (offsets, order, src_sorted.contiguous(), dst_sorted.contiguous(), src_offsets,
                src_order)
        self._cache[key] = plan
        self._lru.append(key)
        while len(self._lru) > self._capacity:
            self._cache.pop(self._lru.pop(0), None)
        return plan


@dataclass
class _Session:
    ops: Any
    stats: FusedStats
    reference_softmax: Any
    csr: _CsrView = field(default_factory=_CsrView)
    warned: bool = False
    force_plan: _ForcePlan | None = None

    # -- softmax seam ---------------------------------------------------------
    def softmax(self, logits, edge_env, dst, n_nodes, z_bias_raw, eps, src_weight=None):
        stats = self.stats

        def stock(weight=None):
            stats.softmax_fallbacks += 1
            return self.reference_softmax(logits, edge_env, dst, n_nodes, z_bias_raw, eps, weight)

        if src_weight is not None:
            return stock(src_weight)
        shaped = (
            _usable_tensor(logits)
            and logits.ndim == 3
            and logits.shape[0] > 0
            and _usable_tensor(edge_env)
            and isinstance(dst, torch.Tensor)
            and dst.dtype == torch.int64
            and dst.ndim == 1
            and n_nodes > 0
        )
        if not shaped:
            return stock()
        n_edges, n_focus, n_head = logits.shape
        channels = n_focus * n_head
        bias = z_bias_raw.to(dtype=torch.float32).reshape(-1)
        if bias.numel() != channels or edge_env.numel() != n_edges:
            return stock()
        try:
            offsets, order = self.csr.get(dst, n_nodes)
            null = torch.log(F.softplus(bias) + float(eps))
            null = null.reshape(1, channels).expand(n_nodes, channels).contiguous()
            result = self.ops.segment_softmax(
                logits.reshape(n_edges, channels),
                edge_env.reshape(n_edges),
                offsets,
                null,
                order=order,
            )
            # (alpha, null_alpha) when a null logit is given; accept a bare
            # tensor too so the seam does not depend on that arity.
            alpha = result[0] if isinstance(result, tuple) else result
        except Exception as error:  # noqa: BLE001 - fall back, never break inference
            self._record(error)
            return stock()
        stats.softmax_hits += 1
        return alpha.reshape(n_edges, n_focus, n_head)

    # -- envelope seam --------------------------------------------------------
    def envelope(self, original, block, x, edge_cache, radial_feat):
        stats = self.stats

        def stock():
            stats.envelope_fallbacks += 1
            return original(x, edge_cache, radial_feat)  # bound to `block` already

        dst = getattr(edge_cache, "dst", None)
        edge_env = getattr(edge_cache, "edge_env", None)
        inverse = getattr(edge_cache, "inv_sqrt_deg", None)
        gate = getattr(edge_cache, "edge_src_gate", None)
        ready = (
            not bool(getattr(block, "training", False))
            and _usable_tensor(x)
            and _usable_tensor(edge_env)
            and _usable_tensor(inverse)
            and isinstance(dst, torch.Tensor)
            and dst.dtype == torch.int64
            and dst.ndim == 1
            and dst.numel() > 0
            and (gate is None or _usable_tensor(gate))
        )
        if not ready:
            return stock()
        n_node, n_edges = x.shape[0], dst.shape[0]
        if (
            x.ndim != 3
            or inverse.numel() != n_node
            or edge_env.numel() != n_edges
            or not _usable_tensor(dst, dtype=torch.int64)
        ):
            return stock()
        try:
            message, _ = block.edge_message(x, edge_cache, radial_feat)
            if not _usable_tensor(message) or message.shape[0] != n_edges:
                raise ValueError("edge message is not a contiguous fp32 (E, ...) tensor")
            weight = edge_env.reshape(-1)
            if gate is not None:
                weight = weight * gate.reshape(-1).to(dtype=torch.float32)
            offsets, order = self.csr.get(dst, n_node)
            out = self.ops.segment_sum(
                message.reshape(n_edges, -1),
                dst,
                offsets,
                weight.contiguous(),
                inverse.reshape(-1).contiguous(),
                order=order,
            )
        except Exception as error:  # noqa: BLE001 - fall back, never break inference
            self._record(error)
            return stock()
        stats.envelope_hits += 1
        return out.reshape(x.shape)

    # -- force seam -----------------------------------------------------------
    def force(self, original, g, edge_vec, src, dst, n_ext):
        """``(force [n_ext, 3], atom_virial [n_ext, 9])`` of an edge list.

        ``g`` is dE/d(edge_vec) per edge with ``edge_vec = r_src - r_dst``, so
        ``F_k = sum_{dst=k} g - sum_{src=k} g`` and the per-atom virial is
        ``-sum_{src=k} g (x) edge_vec`` (row-major), the four ``index_add_``
        scatters of DeepMD's post-processing step
        (``docs/fused-operators.md:111-140`` of the reference).  Ghost atoms
        are rows like any other: folding them onto their local images stays
        with DeepMD.
        """
        stats = self.stats

        def stock():
            stats.force_fallbacks += 1
            return original(g, edge_vec, src, dst, n_ext)

        ready = (
            _usable_tensor(g)
            and _usable_tensor(edge_vec)
            and g.ndim == 2
            and g.shape[1] == 3
            and g.shape[0] > 0
            and tuple(edge_vec.shape) == tuple(g.shape)
            and _usable_tensor(src, dtype=torch.int64)
            and _usable_tensor(dst, dtype=torch.int64)
            and tuple(src.shape) == (g.shape[0],)
            and tuple(dst.shape) == (g.shape[0],)
            and int(n_ext) > 0
            and not g.requires_grad
        )
        if not ready:
            return stock()
        try:
            if self.force_plan is None:
                self.force_plan = _ForcePlan(self.csr, getattr(self.ops, "group_by_source", None))
            offsets, order, src_s, dst_s, src_offsets, src_order = self.force_plan.get(
                src, dst, int(n_ext))
            if order is not None:
                g = g.index_select(0, order)
                edge_vec = edge_vec.index_select(0, order)
            force, virial = self.ops.force_assembly(g, edge_vec, src_s, dst_s, offsets,
                                                    src_offsets, src_order)
        except Exception as error:  # noqa: BLE001 - fall back, never break inference
            self._record(error)
            return stock()
        stats.force_hits += 1
        return force, virial

    def _record(self, error: Exception) -> None:
        self.stats.last_error = f"{type(error).__name__}: {error}"
        if not self.warned:
            self.warned = True
            warnings.warn(
                "fused DeepMD dispatch fell back to the reference path: " + self.stats.last_error,
                RuntimeWarning,
                stacklevel=3,
            )


_SESSION: _Session | None = None
# "<module>.segment_envelope_gated_softmax" -> (module, original callable)
# "block:<id>"                               -> (block, original bound method)
_SAVED: dict[str, Any] = {}


def _softmax_namespaces() -> list[Any]:
    """DeepMD modules whose ``segment_envelope_gated_softmax`` is rebound."""
    import deepmd.pt.model.descriptor.sezm_nn.attention as attention_module
    import deepmd.pt.model.descriptor.sezm_nn.so2 as so2_module

    found = [attention_module, so2_module]
    try:
        import deepmd.pt.model.descriptor.sezm_nn as package
    except ImportError:  # pragma: no cover - the package exists with its modules
        return found
    found.append(package)
    return found


def _force_namespaces() -> list[Any]:
    """DeepMD modules whose ``edge_force_virial`` is rebound (none if absent)."""
    try:
        import deepmd.pt.model.model.transform_output as transform_output
    except ImportError:
        return []
    return [transform_output]


def _blocks(model: Any) -> list[Any]:
    """SO(2) convolution blocks that carry the aggregation seams."""
    return [
        module
        for module in model.modules()
        if callable(getattr(module, "edge_message", None))
        and callable(getattr(module, "forward_envelope", None))
        and hasattr(module, "_segment_softmax_fn")
    ]


def _module_root(model: Any) -> tuple[Any | None, str]:
    """The ``nn.Module`` tree behind a ``DeepPot`` / ``DeepEval`` wrapper.

    ``DeepPot`` is not a module: the legacy ``pt`` backend keeps its tree at
    ``deep_eval.dp``, ``pt_expt`` at ``deep_eval._dpmodel``; a module may also
    be passed directly.
    """
    if callable(getattr(model, "modules", None)):
        return model, "model"
    deep_eval = getattr(model, "deep_eval", None)
    if deep_eval is None:
        return None, ""
    for attribute in ("_dpmodel", "dp", "model"):
        candidate = getattr(deep_eval, attribute, None)
        if candidate is not None and callable(getattr(candidate, "modules", None)):
            return candidate, f"deep_eval.{attribute}"
    if callable(getattr(deep_eval, "modules", None)):
        return deep_eval, "deep_eval"
    return None, ""


def describe_module(module: Any, *, max_depth: int = 2, max_rows: int = 40) -> list[str]:
    """Printable lines: the module tree (to ``max_depth``) and the patch targets."""
    root, path = _module_root(module)
    if root is None:
        return [
            f"module: {type(module).__name__} (no nn.Module tree found -- expected a "
            "module, or a DeepPot/DeepEval wrapper with deep_eval.dp / deep_eval._dpmodel)",
            "patch targets: 0 (nothing can be bound)",
        ]
    named = list(root.named_modules()) if hasattr(root, "named_modules") else []
    via = "" if path == "model" else f" -> {path}"
    lines = [f"module: {type(module).__name__}{via} ({type(root).__name__}, {len(named)} submodules)"]
    for name, child in named[:max_rows]:
        depth = name.count(".") + 1 if name else 0
        if depth <= max_depth:
            lines.append(f"  {'  ' * depth}{name or '<root>'}  {type(child).__name__}")
    if len(named) > max_rows:
        lines.append(f"  ... {len(named) - max_rows} more submodules")
    targets = _blocks(root)
    lines.append(f"patch targets: {len(targets)} SO(2) block(s)")
    for index, block in enumerate(targets):
        lines.append(
            f"  [{index}] {type(block).__name__}  "
            f"n_atten_head={getattr(block, 'n_atten_head', '?')}  "
            "seams: forward_envelope -> segment_sum, attention softmax -> segment_softmax"
        )
    return lines


def _say(verbose: bool, text: str) -> None:
    if verbose:
        print(f"[deepmd_patch] {text}", flush=True)


def deepmd_patch(module: Any, *, ops: Any = None, softmax: bool = True, envelope: bool = True,
                 blocks: Iterable[Any] | None = None, namespaces: Iterable[Any] | None = None,
                 verbose: bool = True, force: bool = False,
                 force_namespaces: Iterable[Any] | None = None) -> FusedStats:
    """Bind the fused operators on ``module`` (a ``DeepPot`` or an ``nn.Module``).

    ``ops`` is an operator bundle with ``segment_softmax`` and ``segment_sum``
    (and optionally ``segment_offsets`` / ``destination_csr`` for the CSR
    view, ``force_assembly`` and ``group_by_source`` for the force seam); it
    defaults to :mod:`bysj_b200.kernels`, and the install is a logged no-op
    when the extension cannot run on this host.  ``namespaces`` overrides the
    DeepMD modules that carry the softmax name, ``force_namespaces`` those
    that carry ``edge_force_virial`` (the third seam, off unless ``force``).
    Installing twice keeps one patch.
    """
    global _SESSION
    stats = FusedStats()
    if verbose:
        for line in describe_module(module):
            _say(True, line)
    uninstall(module)
    root, path = _module_root(module)
    if blocks is not None:
        targets = list(blocks)
    else:
        targets = [] if root is None else list(_blocks(root))
    if root is not None and path != "model":
        _say(verbose, f"resolved module tree: {path} ({type(root).__name__})")
    stats.blocks = len(targets)
    if ops is None:
        ops = _load_ops()
    _say(verbose, f"operators: {'bysj_b200.kernels' if ops is not None else 'unavailable'}; "
                  f"softmax={softmax} envelope={envelope}")
    if ops is None:
        _say(verbose, "no fused extension on this host -> nothing replaced")
        return stats

    spaces: list[Any] = []
    reference = None
    if softmax:
        spaces = list(namespaces) if namespaces is not None else _softmax_namespaces()
        if not spaces:
            raise ValueError("deepmd_patch requires one module namespace to patch")
        reference = getattr(spaces[0], _SOFTMAX_NAME)
    builder = getattr(ops, "segment_offsets", None)
    _SESSION = _Session(ops=ops, stats=stats, reference_softmax=reference,
                        csr=_CsrView(builder, csr=getattr(ops, "destination_csr", None)))

    if softmax:
        def bound_softmax(logits, edge_env, dst, n_nodes, z_bias_raw, eps, src_weight=None):
            session = _SESSION
            if session is None:  # uninstalled between calls
                return reference(logits, edge_env, dst, n_nodes, z_bias_raw, eps, src_weight)
            return session.softmax(logits, edge_env, dst, n_nodes, z_bias_raw, eps, src_weight)

        for space in spaces:
            if not hasattr(space, _SOFTMAX_NAME):
                continue
            _SAVED[f"{space.__name__}.{_SOFTMAX_NAME}"] = (space, getattr(space, _SOFTMAX_NAME))
            setattr(space, _SOFTMAX_NAME, bound_softmax)
            _say(verbose, f"replace {space.__name__}.{_SOFTMAX_NAME} -> "
                          "bysj_b200.model.fused_deepmd.bound_softmax")
        stats.bound_softmax = True

    if envelope:
        for block in targets:
            original = block.forward_envelope
            _SAVED[f"{_BLOCK_PREFIX}{id(block)}"] = (block, original)

            def patched(self, x, edge_cache, radial_feat, _original=original):
                # `_original` is the block's bound method captured at install.
                session = _SESSION
                if session is None:
                    return _original(x, edge_cache, radial_feat)
                return session.envelope(_original, self, x, edge_cache, radial_feat)

            block.forward_envelope = MethodType(patched, block)
        stats.bound_envelope = bool(targets)
        _say(verbose, f"replace SO2Convolution.forward_envelope on {len(targets)} block(s) -> "
                      "bysj_b200.model.fused_deepmd.patched")
    if force:
        force_spaces = (list(force_namespaces) if force_namespaces is not None
                        else _force_namespaces())
        for space in force_spaces:
            if not hasattr(space, _FORCE_NAME):
                _say(verbose, f"{getattr(space, '__name__', space)} has no {_FORCE_NAME}: "
                              "force seam not bound there")
                continue
            stock_force = getattr(space, _FORCE_NAME)
            _SAVED[f"{space.__name__}.{_FORCE_NAME}"] = (space, stock_force)

            def bound_force(g, edge_vec, src, dst, n_ext, _stock=stock_force):
                session = _SESSION
                if session is None:
                    return _stock(g, edge_vec, src, dst, n_ext)
                return session.force(_stock, g, edge_vec, src, dst, n_ext)

            setattr(space, _FORCE_NAME, bound_force)
            stats.bound_force = True
            _say(verbose, f"replace {space.__name__}.{_FORCE_NAME} -> "
                          "bysj_b200.model.fused_deepmd.bound_force")
    _say(verbose, f"installed: softmax={stats.bound_softmax} envelope={stats.bound_envelope} "
                  f"force={stats.bound_force} blocks={stats.blocks}")
    return stats


def uninstall(module: Any = None) -> None:
    """Restore every rebound name; safe to call when nothing is installed."""
    global _SESSION
    for key, (owner, original) in list(_SAVED.items()):
        if key.startswith(_BLOCK_PREFIX):
            # Drop the instance attribute so the class method shows through.
            owner.__dict__.pop("forward_envelope", None)
        else:
            setattr(owner, key.rsplit(".", 1)[-1], original)
    _SAVED.clear()
    _SESSION = None


def status(stats: FusedStats | None) -> dict[str, Any]:
    """Counters of a patch (empty when it never ran)."""
    return {} if stats is None else stats.as_dict()


__all__ = ["FusedStats", "deepmd_patch", "describe_module", "status", "uninstall"]
