"""Host-side checks of the quantized backends and the shared expert (no GPU).

``QuantizedB200Backend(mode)`` validates a ``QuantizedStore`` bank the way the
reference's ``QuantizedStore.validate`` does (quantized_model.py:45-68) before
any launch; these run on CPU tensors, so they stop before the library is used.
"""

from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

from drama_b200 import synthetic
from drama_b200.backend import QUANTIZED_MODES, QuantizedB200Backend, _w8a8_bank


def test_quantized_modes_and_names():
    assert QUANTIZED_MODES == {0: "W4A16-GPTQ", 1: "INT8-ConvRot", 2: "W6A8", 3: "W4A8"}
    for mode in range(4):
        backend = QuantizedB200Backend(mode)
        assert backend.mode == mode and backend.quantized_mode == QUANTIZED_MODES[mode]
    with pytest.raises(ValueError, match="Unknown quantized bank format"):
        QuantizedB200Backend(4)


@pytest.mark.parametrize("mode", [1, 2, 3])
def test_w8a8_bank_geometry(mode):
    bank = synthetic.w8a8_bank(mode, 2, 256, 256, seed=mode)
    staged = SimpleNamespace(**bank)
    desc, keep = _w8a8_bank(staged, 256, mode)
    assert (desc.mode, desc.slots, desc.hidden, desc.intermediate) == (mode, 2, 256, 256)
    cols = {1: 256, 2: 192, 3: 128}[mode]
    assert desc.w13_row_stride == cols and desc.w13_slot_stride == 512 * cols
    scale_row = {1: 4, 2: 256 // 16 + 4, 3: 256 // 16 + 8}[mode]
    assert desc.w13_scale_row_stride == scale_row
    bad = SimpleNamespace(**{**bank, "w2_weight": bank["w2_weight"][:, :, :-8].contiguous()})
    with pytest.raises(ValueError, match="geometry mismatch"):
        _w8a8_bank(bad, 256, mode)
    wrong = SimpleNamespace(**{**bank, "w13_scale_inv": bank["w13_scale_inv"].to(torch.float64)})
    with pytest.raises(ValueError, match="scale dtype mismatch"):
        _w8a8_bank(wrong, 256, mode)


def test_w8a8_needs_bf16_rows():
    bank = synthetic.w8a8_bank(1, 2, 256, 256, seed=1)
    x = torch.zeros(1, 256, dtype=torch.float16)
    ids = torch.zeros(1, 2, dtype=torch.int64)
    with pytest.raises(ValueError, match="bfloat16 hidden rows"):
        QuantizedB200Backend(1).forward(x, ids, torch.ones(1, 2), SimpleNamespace(**bank))


def test_shared_expert_refuses_host_tensors():
    from drama_b200.shared import SharedExpertB200

    w = torch.zeros(128, 256, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA tensors"):
        SharedExpertB200(w, w, w.t().contiguous(), torch.zeros(1, 256, dtype=torch.bfloat16))
