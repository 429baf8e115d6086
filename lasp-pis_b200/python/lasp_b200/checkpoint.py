"""Seeded synthetic MH1 checkpoint in PyTorch's ZIP format (``torch.save`` of a module tree).

The real MH1 foundation checkpoint is not available, so this writes a stand-in with the
structure the native converter reads (mace/src/weights.cpp:305-393): a six-head, two-layer
``mace.modules.models ScaleShiftMACE`` whose attributes, child modules, e3nn irreps,
linear / tensor-product instructions, radial MLPs and symmetric-contraction coupling
tensors have MH1's names and shapes, with seeded random weights.

Pickle records a class by module and name only.  The stand-in classes below are registered
under MACE's and e3nn's module names for the duration of ``torch.save`` and removed
afterwards; nothing imports MACE or e3nn, and the file is never unpickled in Python.
"""
from __future__ import annotations

import collections
import contextlib
import sys
import types
from pathlib import Path

import numpy as np
import torch

from . import synth

HEADS = ("synthetic_pbe", "matpes_r2scan", "synthetic_pbesol", "synthetic_wb97m", "synthetic_rpbe",
         "synthetic_scan")
SEED = 20261202


# ----------------------------------------------------------------------------- stand-ins

class _Irrep(tuple):
    __slots__ = ()

    def __new__(cls, l, p=None):
        if p is None:  # rebuilt from its pickled form Irrep((l, p))
            l, p = l
        return super().__new__(cls, (l, p))


class _MulIr(tuple):
    __slots__ = ()

    def __new__(cls, mul, ir=None):
        if ir is None:  # rebuilt from its pickled form _MulIr((mul, ir))
            mul, ir = mul
        return super().__new__(cls, (mul, ir))


class _Irreps(tuple):
    """e3nn Irreps: a tuple of (mul, (l, parity)); pickles as Irreps((...,)) like e3nn's.
    Built from (mul, l, parity) triples, or rebuilt from its own elements."""
    __slots__ = ()

    def __new__(cls, blocks):
        return super().__new__(cls, tuple(b if isinstance(b, _MulIr) else _MulIr(b[0], _Irrep(b[1], b[2]))
                                          for b in blocks))


_LinearInstruction = collections.namedtuple("Instruction", "i_in i_out path_shape path_weight")
_TPInstruction = collections.namedtuple(
    "Instruction", "i_in1 i_in2 i_out connection_mode has_weight path_weight path_shape")


class _Module(torch.nn.Module):
    """A module with the given plain attributes, parameters, buffers and children."""

    def __init__(self, attrs=None, params=None, buffers=None, children=None):
        super().__init__()
        for k, v in (attrs or {}).items():
            setattr(self, k, v)
        for k, v in (params or {}).items():
            self.register_parameter(k, torch.nn.Parameter(v, requires_grad=False))
        for k, v in (buffers or {}).items():
            self.register_buffer(k, v)
        for k, v in (children or {}).items():
            self.add_module(k, v)


# (module name, class name) -> stand-in class.  Classes that only carry data get a fresh
# subclass of _Module so that their pickled label is the MACE / e3nn name.
_NAMES = {
    "mace.modules.models": ["ScaleShiftMACE"],
    "mace.modules.blocks": ["LinearNodeEmbeddingBlock", "RadialEmbeddingBlock",
                            "RealAgnosticResidualNonLinearInteractionBlock",
                            "EquivariantProductBasisBlock", "LinearReadoutBlock",
                            "NonLinearReadoutBlock", "AtomicEnergiesBlock", "ScaleShiftBlock"],
    "mace.modules.radial": ["BesselBasis", "PolynomialCutoff", "AgnesiTransform", "ZBLBasis",
                            "RadialMLP"],
    "mace.modules.symmetric_contraction": ["SymmetricContraction", "Contraction"],
    "e3nn.o3._linear": ["Linear"],
    "e3nn.o3._tensor_product._tensor_product": ["TensorProduct"],
    "e3nn.nn._gate": ["Gate"],
    "e3nn.nn._activation": ["Activation"],
    "e3nn.math._normalize_activation": ["normalize2mom"],
}
_CLASSES = {name: type(name, (_Module,), {"__module__": module, "__qualname__": name})
            for module, names in _NAMES.items() for name in names}
_EXTRA = {
    "e3nn.o3._irreps": {"Irreps": _Irreps, "Irrep": _Irrep, "_MulIr": _MulIr},
    "e3nn.o3._linear": {"Instruction": _LinearInstruction},
    "e3nn.o3._tensor_product._instruction": {"Instruction": _TPInstruction},
}
for _module, _members in _EXTRA.items():
    for _name, _cls in _members.items():
        _cls.__module__, _cls.__qualname__ = _module, _name


@contextlib.contextmanager
def _registered():
    """Make the stand-ins importable under their MACE / e3nn names while saving."""
    members: dict[str, dict[str, type]] = {}
    for module, names in _NAMES.items():
        members.setdefault(module, {}).update({n: _CLASSES[n] for n in names})
    for module, extra in _EXTRA.items():
        members.setdefault(module, {}).update(extra)
    wanted = set()
    for module in members:
        parts = module.split(".")
        wanted.update(".".join(parts[:k]) for k in range(1, len(parts) + 1))
    saved = {m: sys.modules.get(m) for m in wanted}
    try:
        for m in sorted(wanted):
            sys.modules[m] = types.ModuleType(m)
        for module, names in members.items():
            for n, cls in names.items():
                setattr(sys.modules[module], n, cls)
        yield
    finally:
        for m, old in saved.items():
            if old is None:
                sys.modules.pop(m, None)
            else:
                sys.modules[m] = old


# ----------------------------------------------------------------------------- building

class _Builder:
    def __init__(self, seed: int, dtype: torch.dtype):
        self.rng = np.random.default_rng(seed)
        self.dtype = dtype

    def t(self, a) -> torch.Tensor:
        return torch.tensor(np.asarray(a, np.float64), dtype=self.dtype)

    def normal(self, *shape, scale=1.0) -> torch.Tensor:
        return self.t(self.rng.normal(size=shape) * scale)

    def linear(self, ins, outs) -> torch.nn.Module:
        """e3nn o3.Linear between (mul, l, parity) block lists, element path normalisation."""
        pairs = [(i, o) for i, (_, li, pi) in enumerate(ins) for o, (_, lo, po) in enumerate(outs)
                 if (li, pi) == (lo, po)]
        fan = collections.Counter()
        for i, o in pairs:
            fan[o] += ins[i][0]
        inst = [_LinearInstruction(i, o, (ins[i][0], outs[o][0]), float(fan[o]) ** -0.5) for i, o in pairs]
        weight = self.normal(sum(ins[i][0] * outs[o][0] for i, o in pairs))
        return _CLASSES["Linear"](attrs={"irreps_in": _Irreps(ins), "irreps_out": _Irreps(outs),
                                         "instructions": inst},
                                  params={"weight": weight})

    def radial_mlp(self, depth: int, outputs: int) -> torch.nn.Module:
        layers = []
        for k in range(depth):
            fan = 1034 if k == 0 else 64
            lin = torch.nn.Linear(fan, 64, dtype=self.dtype)
            norm = torch.nn.LayerNorm(64, eps=1e-5, dtype=self.dtype)
            with torch.no_grad():
                lin.weight.copy_(self.normal(64, fan, scale=fan ** -0.5))
                lin.bias.copy_(self.normal(64, scale=0.1))
                norm.weight.copy_(1 + self.normal(64, scale=0.1))
                norm.bias.copy_(self.normal(64, scale=0.1))
            layers += [lin, norm, torch.nn.SiLU()]
        out = torch.nn.Linear(64, outputs, dtype=self.dtype)
        with torch.no_grad():
            out.weight.copy_(self.normal(outputs, 64, scale=1 / 8))
            out.bias.copy_(self.normal(outputs, scale=0.1))
        return _CLASSES["RadialMLP"](children={"net": torch.nn.Sequential(*layers, out)})

    def tensor_product(self, layer: int, up, message_order) -> torch.nn.Module:
        paths, out_start, _, _ = synth.tp_layout(layer)
        sh = [(1, l, synth.PARITY[l]) for l in range(4)]
        message = [(128, paths[p][2], synth.PARITY[paths[p][2]]) for p in message_order]
        inst = []
        for p, (li, ls, lo) in enumerate(paths):
            inst.append(_TPInstruction(li, ls, message_order.index(p), "uvu", True,
                                       float(np.sqrt((2 * lo + 1) / (1 + layer))), (128, 1)))
        return _CLASSES["TensorProduct"](attrs={"irreps_in1": _Irreps(up), "irreps_in2": _Irreps(sh),
                                                "irreps_out": _Irreps(message), "instructions": inst})

    def contraction(self, out_l: int) -> torch.nn.Module:
        coupling = synth._coupling_paths(out_l)
        buffers, weights = {}, {}
        for degree in (1, 2, 3):
            # Rounded to 1e-12 so that the last bits of the numerical 3j symbols (SVD based)
            # cannot change the file between machines.
            u = np.round(np.stack(coupling[degree], axis=-1), 12)
            if out_l == 0:
                u = u[0]
            buffers[f"U_matrix_{degree}"] = self.t(u)
            n = u.shape[-1]
            weights[degree] = self.normal(1, n, 512, scale=(1.0, 0.3, 0.05)[degree - 1] / np.sqrt(n))
        plist = torch.nn.ParameterList([torch.nn.Parameter(weights[2], requires_grad=False),
                                        torch.nn.Parameter(weights[1], requires_grad=False)])
        return _CLASSES["Contraction"](attrs={"correlation": 3},
                                       params={"weights_max": weights[3]}, buffers=buffers,
                                       children={"weights": plist})

    def activation(self, cst: float) -> torch.nn.Module:
        act = _CLASSES["normalize2mom"](attrs={"f": torch.nn.functional.silu, "cst": cst})
        return _CLASSES["Activation"](children={"acts": torch.nn.ModuleList([act])})


def build_model(seed: int = SEED, dtype: torch.dtype = torch.float64,
                species=synth.SPECIES) -> torch.nn.Module:
    """The ScaleShiftMACE-shaped module tree, seeded."""
    b = _Builder(seed, dtype)
    s = len(species)
    c = [6.0, np.sqrt(2.0 / 6.0), 5.0, 1.0805, 0.9183, 4.5791, 0.8, -0.05, 0.300, 0.4543, 6.0,
         1.6790, 1.8484, 1.6790]
    scalar = [(512, 0, 1)]
    pre = [(2048, 0, 1), (512, 1, -1), (512, 2, 1), (512, 3, -1)]
    gated = [(512, l, synth.PARITY[l]) for l in range(4)]
    hidden = [[(512, 0, 1), (512, 1, -1)], [(512, 0, 1)]]
    one_hot = [(s, 0, 1)]

    def embedding():
        return b.linear(one_hot, scalar)

    interactions, products = [], []
    for layer in range(2):
        node = scalar if layer == 0 else hidden[0]
        up = [(128, 0, 1)] if layer == 0 else [(128, 0, 1), (128, 1, -1)]
        paths, out_start, _, _ = synth.tp_layout(layer)
        order = sorted(out_start, key=out_start.get)
        message = [(128, paths[p][2], synth.PARITY[paths[p][2]]) for p in order]
        gate = _CLASSES["Gate"](children={"act_scalars": b.activation(c[11]),
                                          "act_gates": b.activation(c[12])})
        interactions.append(_CLASSES["RealAgnosticResidualNonLinearInteractionBlock"](
            params={"alpha": b.t(1.0 + 0.1 * layer), "beta": b.t(0.9 + 0.05 * layer)},
            children={
                "source_embedding": embedding(), "target_embedding": embedding(),
                "linear_up": b.linear(node, up), "linear_res": b.linear(up, pre),
                "conv_tp_weights": b.radial_mlp(3, len(paths) * 128),
                "density_fn": b.radial_mlp(1, 1),
                "conv_tp": b.tensor_product(layer, up, order),
                "linear_1": b.linear(message, pre), "linear_2": b.linear(gated, gated),
                "skip_tp": b.linear(node, hidden[layer]),
                "equivariant_nonlin": gate,
            }))
        contractions = [b.contraction(0)] + ([b.contraction(1)] if layer == 0 else [])
        products.append(_CLASSES["EquivariantProductBasisBlock"](children={
            "symmetric_contractions": _CLASSES["SymmetricContraction"](
                children={"contractions": torch.nn.ModuleList(contractions)}),
            "linear": b.linear(hidden[layer], hidden[layer]),
        }))
    heads = len(HEADS)
    readouts = [
        _CLASSES["LinearReadoutBlock"](children={"linear": b.linear(hidden[0], [(heads, 0, 1)])}),
        _CLASSES["NonLinearReadoutBlock"](children={
            "linear_1": b.linear(hidden[1], [(16 * heads, 0, 1)]),
            "non_linearity": b.activation(c[13]),
            "linear_2": b.linear([(16 * heads, 0, 1)], [(heads, 0, 1)]),
        }),
    ]
    radial = _CLASSES["RadialEmbeddingBlock"](
        attrs={"apply_cutoff": False},
        children={
            "bessel_fn": _CLASSES["BesselBasis"](
                params={"bessel_weights": b.t(np.arange(1, 11) * np.pi / 6.0)},
                buffers={"prefactor": b.t(c[1]), "r_max": b.t(c[0])}),
            "cutoff_fn": _CLASSES["PolynomialCutoff"](buffers={"p": b.t(c[2]), "r_max": b.t(c[0])}),
            "distance_transform": _CLASSES["AgnesiTransform"](buffers={
                "a": b.t(c[3]), "q": b.t(c[4]), "p": b.t(c[5]),
                "covalent_radii": b.t(b.rng.uniform(0.5, 1.6, size=119))}),
        })
    zbl = _CLASSES["ZBLBasis"](
        params={"a_exp": b.t(c[8]), "a_prefactor": b.t(c[9])},
        buffers={"p": b.t(c[10]), "c": b.t([0.1818, 0.5099, 0.2802, 0.02817]),
                 "covalent_radii": b.t(b.rng.uniform(0.5, 1.1, size=119))})
    return _CLASSES["ScaleShiftMACE"](
        attrs={"heads": list(HEADS)},
        buffers={"r_max": b.t(c[0]), "atomic_numbers": torch.tensor(species, dtype=torch.int64)},
        children={
            "node_embedding": _CLASSES["LinearNodeEmbeddingBlock"](children={"linear": embedding()}),
            "radial_embedding": radial,
            "pair_repulsion_fn": zbl,
            "atomic_energies_fn": _CLASSES["AtomicEnergiesBlock"](
                buffers={"atomic_energies": b.t(b.rng.uniform(-10, -1, size=(heads, s)))}),
            "scale_shift": _CLASSES["ScaleShiftBlock"](buffers={
                "scale": b.t(b.rng.uniform(0.6, 1.0, size=heads)),
                "shift": b.t(b.rng.uniform(-0.1, 0.1, size=heads))}),
            "interactions": torch.nn.ModuleList(interactions),
            "products": torch.nn.ModuleList(products),
            "readouts": torch.nn.ModuleList(readouts),
        })


def save(model: torch.nn.Module, path: str | Path) -> Path:
    """torch.save the stand-in module tree (PyTorch ZIP format, pickle protocol 2)."""
    path = Path(path)
    with _registered():
        torch.save(model, path)
    return path


def write_checkpoint(path: str | Path, seed: int = SEED, dtype: torch.dtype = torch.float64) -> Path:
    return save(build_model(seed, dtype), path)


if __name__ == "__main__":
    import argparse

    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("output")
    p.add_argument("--seed", type=int, default=SEED)
    p.add_argument("--dtype", choices=("float32", "float64"), default="float64")
    a = p.parse_args()
    write_checkpoint(a.output, a.seed, getattr(torch, a.dtype))
