"""The inference load on the GPU: a .plx written by the reference's
pack._write_plx (tests/golden/tiny.plx) parsed from an mmap straight into
device tensors through page-locked staging (read_plx(device="cuda"), the
reader of generate.py:76-136), then every packed H24 layer materialised with
one batched dequant launch (materialize_all; PolluxModel.from_packed_checkpoint,
pollux.py:704-752) and compared bit for bit with the oracle's dequant of the
same bytes and with the host-parsed tensors."""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN

pytestmark = pytest.mark.gpu


def test_plx_gpu_direct_load_and_materialize(lib, oracle):
    from pollux_b200 import packed_linear, plx
    path = os.path.join(GOLDEN, "tiny.plx")
    host = plx.read_plx(path)
    dev = plx.read_plx(path, device="cuda")
    assert list(dev["state_dict"]) == list(host["state_dict"])
    for k, t in dev["state_dict"].items():
        assert t.device.type == "cuda" and torch.equal(t.cpu(), host["state_dict"][k]), k
    layers = {}
    for name, t in dev["state_dict"].items():
        if name.endswith(".packed_weights"):
            base = name[: -len(".packed_weights")]
            s = dev["state_dict"][base + ".sigma_rows"]
            rows = s.numel()
            in_f = (t.numel() // 9) * 4 * 24 // rows
            m = packed_linear.PackedH24Linear(in_f, rows).cuda()
            m.packed_weights = t
            m.sigma_rows = s
            layers[base] = m
    assert layers, "the fixture holds a packed H24 layer"
    model = torch.nn.ModuleDict({k.replace(".", "_"): m for k, m in layers.items()})
    assert packed_linear.materialize_all(model) == len(layers)
    for base, m in layers.items():
        p = host["state_dict"][base + ".packed_weights"].numpy()
        s = host["state_dict"][base + ".sigma_rows"].numpy()
        want = oracle.dequant(p, s, m.out_features, m.in_features)
        got = m.weight.detach().cpu().numpy()
        assert got.dtype == np.float16
        assert np.array_equal(got.view(np.uint16), want.view(np.uint16)), base
