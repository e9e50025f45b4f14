"""mkb_ln_modulate against the oracle's ln_modulate (src/kernels/image.metal:33-53 plus the optional shift): bf16
output within 1e-2 of the output scale, for every kernel instance (n 640 to 4096), ragged row counts and the
split between two modulation rows; and bad widths are rejected."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_ln_modulate_oracle(cuda):
    from oracle import ops as O
    import ln_cases

    got, status = ln_cases.run(cuda)
    assert status == 0
    for (rows, n, split, ws), x, mod, shift in ln_cases.inputs("cpu"):
        x, mod = x.numpy(), mod.numpy()
        sel = np.where(np.arange(rows)[:, None] < split, 1, 0)  # rows before split take modulation row 1
        scale = mod[sel[:, 0]]
        sh = shift.numpy()[sel[:, 0]] if shift is not None else None
        ref = O.ln_modulate(x, scale, sh, eps=1e-6)
        y = got[f"ln_{rows}x{n}_{split}_{int(ws)}"]
        assert np.abs(y - ref).max() < 1e-2 * np.abs(ref).max(), (rows, n)


def test_ln_modulate_rejects(cuda):
    import torch
    import mkimage

    x = torch.zeros(4, 100, device=cuda)
    mod = torch.zeros(2, 128, device=cuda)
    with pytest.raises(mkimage._lib.MkbError):
        mkimage.ops.ln_modulate(x, mod)
