"""DeepMD-backed inference facade that can bind the B200 fused operators.

Same contract as the reference's ``python/model/dpa4.py`` (lines 31-193):
DeepMD-kit owns the DPA4/SeZM graph, checkpoints, neighbour lists, energy,
forces and virial; this facade only adds the ``fused=`` switch (installing the
seams of :mod:`bysj_b200.model.fused_deepmd`) and a close / context-manager
lifecycle that removes them before the underlying ``DeepPot`` is closed.
"""
from __future__ import annotations

import os
from pathlib import Path
from typing import Any

_FUSED_SEAMS = ("softmax", "envelope", "force")
# ``fused=True`` keeps the reference's meaning (its two seams); the force
# seam, which the reference lists as not yet wired, is opt-in by name.
_DEFAULT_SEAMS = ("softmax", "envelope")
_REMOVED_SELECTORS = (
    ("tilelang_ops", "drop the argument; TileLang dispatch was removed from this project"),
    ("native_ops", 'drop the argument and use fused=("softmax", "envelope") instead'),
)


def _normalize_fused(fused: Any) -> dict[str, bool] | None:
    """Translate the ``fused`` switch into per-seam switches (``None``: off)."""
    if not fused:
        return None
    if fused is True:
        return dict.fromkeys(_DEFAULT_SEAMS, True)
    if isinstance(fused, str):
        fused = (fused,)
    if isinstance(fused, (list, tuple, set, frozenset)):
        chosen: dict[str, bool] = {}
        for value in fused:
            name = value.strip().lower() if isinstance(value, str) else None
            if name not in _FUSED_SEAMS:
                raise ValueError(
                    f"unknown fused seam {value!r}; choose from: {', '.join(_FUSED_SEAMS)}"
                )
            chosen[name] = True
        return chosen
    if isinstance(fused, dict):
        unknown = set(fused) - set(_FUSED_SEAMS)
        if unknown:
            raise ValueError(
                f"unknown fused seams: {', '.join(sorted(map(str, unknown)))}; "
                f"choose from: {', '.join(_FUSED_SEAMS)}"
            )
        chosen = {name: bool(fused.get(name, False)) for name in _DEFAULT_SEAMS}
        if "force" in fused:
            chosen["force"] = bool(fused["force"])
        return chosen
    raise TypeError("fused must be a bool, a seam name, a sequence of names or a mapping")


def _create_deep_pot(model_file: str, **kwargs: Any) -> Any:
    """Import DeepMD lazily so importing this facade needs no DeepMD."""
    try:
        from deepmd.infer import DeepPot
    except ImportError as error:
        raise RuntimeError(
            "DPA4Model requires an installed DeepMD-kit with the PyTorch inference backend."
        ) from error
    return DeepPot(model_file, **kwargs)


def _backend_name(deep_pot: Any) -> str:
    module_name = type(getattr(deep_pot, "deep_eval", None)).__module__
    parts = module_name.split(".")
    return parts[1] if len(parts) >= 2 and parts[0] == "deepmd" else "unknown"


class DPA4Model:
    """``DeepPot`` facade that can bind the fused segmented operators.

    ``fused``: ``True`` installs the softmax and envelope seams; a seam name
    or a sequence of names (``"softmax"``, ``"envelope"``, ``"force"``)
    selects some; a mapping sets each;
    ``None`` / ``False`` leaves DeepMD untouched.  Remaining keyword
    arguments go to ``deepmd.infer.DeepPot``.
    """

    def __init__(self, model_file: str | os.PathLike[str], *, fused: Any = None,
                 **deepmd_kwargs: Any) -> None:
        self.model_file = str(Path(model_file).expanduser())
        for removed, hint in _REMOVED_SELECTORS:
            if removed in deepmd_kwargs:
                raise RuntimeError(
                    f"{removed} was removed from DPA4Model: {hint}; an old call site should "
                    "fail loudly instead of being forwarded to DeepPot"
                )
        # Parse the switch before loading, so a typo fails before a large
        # checkpoint is read.
        self.fused_seams = _normalize_fused(fused)
        self._deep_pot = _create_deep_pot(self.model_file, **deepmd_kwargs)
        self.backend = _backend_name(self._deep_pot)
        self.fused_ops: dict[str, Any] = {}
        if self.fused_seams:
            from .fused_deepmd import deepmd_patch, status

            self.fused_ops = dict(status(deepmd_patch(self._deep_pot, **self.fused_seams)))

    def eval(self, coords: Any, cells: Any, atom_types: Any, *, atomic: bool = False,
             fparam: Any = None, aparam: Any = None, **kwargs: Any) -> Any:
        """Energy, forces and virial through DeepMD's public API."""
        return self._deep_pot.eval(coords, cells, atom_types, atomic=atomic, fparam=fparam,
                                   aparam=aparam, **kwargs)

    predict = eval
    __call__ = eval

    def get_rcut(self) -> float:
        return self._deep_pot.get_rcut()

    def get_type_map(self) -> list[str]:
        return self._deep_pot.get_type_map()

    def get_ntypes(self) -> int:
        return self._deep_pot.get_ntypes()

    def get_model_def_script(self) -> Any:
        return self._deep_pot.get_model_def_script()

    def close(self) -> None:
        if self.fused_ops:
            from .fused_deepmd import uninstall

            uninstall(self._deep_pot)
            self.fused_ops = {}
        closer = getattr(self._deep_pot, "close", None)
        if callable(closer):
            closer()

    def __enter__(self) -> "DPA4Model":
        return self

    def __exit__(self, exc_type: Any, exc_value: Any, traceback: Any) -> None:
        self.close()

    def __repr__(self) -> str:
        return (
            f"DPA4Model(model_file={self.model_file!r}, backend={self.backend!r}, "
            f"fused_ops={self.fused_ops!r})"
        )


__all__ = ["DPA4Model"]
