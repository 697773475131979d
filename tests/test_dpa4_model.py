"""Contracts of the DeepMD-backed facade (no GPU, no DeepMD).

Modelled on the reference's ``tests/python/test_dpa4_model.py``: the facade
forwards to ``DeepPot``, parses ``fused=`` before loading anything, installs
and removes the seams, and fails loudly on removed selectors.
"""
from __future__ import annotations

from types import SimpleNamespace
from unittest import mock

import numpy as np
import pytest

from bysj_b200.model import dpa4
from bysj_b200.model.dpa4 import DPA4Model


class _Backend:
    def __init__(self, module_name):
        self.__class__ = type("Backend", (_Backend,), {"__module__": module_name})


class FakeDeepPot:
    def __init__(self, backend="deepmd.pt.infer.deep_eval"):
        self.deep_eval = _Backend(backend)
        self.calls = []
        self.closed = False

    def eval(self, coords, cells, atom_types, **kwargs):
        self.calls.append((coords, cells, atom_types, kwargs))
        return {"energy": 1.0, "force": 2.0, "virial": 3.0}

    def get_rcut(self):
        return 6.0

    def get_type_map(self):
        return ["O", "H"]

    def get_ntypes(self):
        return 2

    def get_model_def_script(self):
        return {"type": "dpa4"}

    def close(self):
        self.closed = True


def model_with(pot, **kwargs):
    with mock.patch.object(dpa4, "_create_deep_pot", return_value=pot):
        return DPA4Model("water.pt", **kwargs)


def test_eval_forwards_every_argument():
    pot = FakeDeepPot()
    model = model_with(pot)
    coords, cells, types = np.zeros((1, 3, 3)), np.zeros((1, 3, 3)), np.zeros((1, 3), dtype=int)
    assert model.eval(coords, cells, types, atomic=True, fparam=[0.5], aparam=[0.1])["energy"] == 1.0
    c, ce, t, kw = pot.calls[0]
    assert c is coords and ce is cells and t is types
    assert kw == {"atomic": True, "fparam": [0.5], "aparam": [0.1]}
    assert model.predict.__func__ is model.eval.__func__
    assert (model.get_rcut(), model.get_type_map(), model.get_ntypes()) == (6.0, ["O", "H"], 2)
    assert model.get_model_def_script() == {"type": "dpa4"}


def test_backend_name():
    assert model_with(FakeDeepPot()).backend == "pt"
    assert model_with(FakeDeepPot("deepmd.pt_expt.infer.deep_eval")).backend == "pt_expt"
    assert model_with(FakeDeepPot("torch")).backend == "unknown"


def test_fused_switch_installs_and_records():
    pot = FakeDeepPot()
    report = {"softmax_hits": 3, "bound_softmax": True}
    with mock.patch.object(dpa4, "_create_deep_pot", return_value=pot), \
            mock.patch("bysj_b200.model.fused_deepmd.deepmd_patch") as patch, \
            mock.patch("bysj_b200.model.fused_deepmd.status", return_value=report):
        model = DPA4Model("water.pt", fused=True)
    patch.assert_called_once_with(pot, softmax=True, envelope=True)
    assert model.fused_ops == report
    assert model.fused_seams == {"softmax": True, "envelope": True}


def test_no_switch_leaves_deepmd_untouched():
    with mock.patch("bysj_b200.model.fused_deepmd.deepmd_patch") as patch:
        model = model_with(FakeDeepPot())
    patch.assert_not_called()
    assert model.fused_ops == {} and model.fused_seams is None


def test_unknown_seam_rejected_before_loading():
    with mock.patch.object(dpa4, "_create_deep_pot") as create:
        with pytest.raises(ValueError, match="unknown fused seam"):
            DPA4Model("water.pt", fused="flash")
    create.assert_not_called()


def test_close_uninstalls_once_and_closes():
    pot = FakeDeepPot()
    with mock.patch.object(dpa4, "_create_deep_pot", return_value=pot), \
            mock.patch("bysj_b200.model.fused_deepmd.deepmd_patch",
                       return_value=SimpleNamespace(as_dict=lambda: {"bound": True})), \
            mock.patch("bysj_b200.model.fused_deepmd.status", return_value={"bound": True}), \
            mock.patch("bysj_b200.model.fused_deepmd.uninstall") as uninstall:
        model = DPA4Model("water.pt", fused=("softmax",))
        model.close()
        assert model.fused_ops == {}
        model.close()
    uninstall.assert_called_once_with(pot)
    assert pot.closed


def test_context_manager_and_repr():
    pot = FakeDeepPot()
    with mock.patch.object(dpa4, "_create_deep_pot", return_value=pot), \
            mock.patch("bysj_b200.model.fused_deepmd.deepmd_patch"), \
            mock.patch("bysj_b200.model.fused_deepmd.status", return_value={"softmax_hits": 1}), \
            mock.patch("bysj_b200.model.fused_deepmd.uninstall"):
        with DPA4Model("water.pt", fused=True) as model:
            text = repr(model)
    assert pot.closed
    assert "backend='pt'" in text and "fused_ops={'softmax_hits': 1}" in text


def test_removed_selectors_fail_loudly():
    for keyword in ("tilelang_ops", "native_ops"):
        with mock.patch.object(dpa4, "_create_deep_pot") as create:
            with pytest.raises(RuntimeError, match=f"{keyword} was removed"):
                DPA4Model("water.pt", **{keyword: ("gie",)})
        create.assert_not_called()


def test_missing_deepmd_is_reported():
    with pytest.raises(RuntimeError, match="DeepMD-kit"):
        DPA4Model("water.pt")
