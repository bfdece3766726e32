"""RoPE kernel (attn_rope) on the GPU against the oracle and the reference's golden vectors."""

import pathlib

import numpy as np
import pytest
import torch

import attnax_b200 as ax
import oracle as O
from tests._util import assert_bf16_close

pytestmark = pytest.mark.gpu
DEV = "cuda"
G = pathlib.Path(__file__).resolve().parent / "golden"


@pytest.mark.parametrize("name,dt,atol", [("f32", torch.float32, 1e-6), ("f16", torch.float16, 8e-3)])
def test_golden_rope(name, dt, atol):
    """The reference's tables and outputs (positions gathered per batch row)."""
    d = dict(np.load(G / "golden_rope.npz"))
    pos = torch.tensor(d["rope_pos"], device=DEV)
    cos, sin = ax.rope_cos_sin_from_positions(pos, 16, 10000.0, 3000, dt)
    x = torch.tensor(d[f"rope_x_{name}"], device=DEV)
    got = ax.apply_rope(x, cos[:, None], sin[:, None])
    np.testing.assert_allclose(got.float().cpu().numpy(), d[f"rope_y_{name}"].astype(np.float32), atol=atol)
    # the same through the tables and position ids (gather fused into the kernel)
    ct = torch.tensor(d[f"rope_cos_{name}"], device=DEV)
    st = torch.tensor(d[f"rope_sin_{name}"], device=DEV)
    got2 = ax.apply_rope_table(x, ct, st, pos)
    np.testing.assert_allclose(got2.float().cpu().numpy(), d[f"rope_y_{name}"].astype(np.float32), atol=atol)


def test_rope_bf16_per_batch_tables_inplace_and_strided():
    rng = np.random.default_rng(3)
    B, H, S, D = 2, 8, 333, 128
    pos = rng.integers(0, 4096, size=(B, S)).astype(np.int32)
    cos, sin = ax.rope_cos_sin_from_positions(torch.tensor(pos, device=DEV), D, 10000.0, 4096, torch.bfloat16)
    x = torch.randn(B, S, H, D, device=DEV).to(torch.bfloat16).transpose(1, 2)  # (B, H, S, D) view, strided
    want = O.apply_rope(x.float().cpu().numpy(), cos.float().cpu().numpy()[:, None], sin.float().cpu().numpy()[:, None])
    got = ax.apply_rope(x, cos[:, None], sin[:, None])
    assert_bf16_close(got.float().cpu().numpy(), want, "bf16 strided")
    y = x.contiguous()
    ax.apply_rope(y, cos[:, None], sin[:, None], out=y)  # in place
    assert_bf16_close(y.float().cpu().numpy(), want, "bf16 in place")


def test_rope_table_positions_wrap_and_clamp():
    """Negative positions count from the end of the table, positions past it clamp."""
    rng = np.random.default_rng(4)
    B, H, S, D, L = 1, 2, 6, 64, 50
    ct, st = ax.rope_cos_sin_table(L, D, 10000.0, torch.float32)
    pos = torch.tensor([[0, 5, -1, -50, 49, 200]], dtype=torch.int32, device=DEV)
    idx = np.array([[0, 5, 49, 0, 49, 49]])
    x = torch.tensor(rng.standard_normal((B, H, S, D)).astype(np.float32), device=DEV)
    got = ax.apply_rope_table(x, ct, st, pos)
    c, s = ct.cpu().numpy()[idx], st.cpu().numpy()[idx]
    want = O.apply_rope(x.cpu().numpy(), c[:, None], s[:, None])
    np.testing.assert_allclose(got.cpu().numpy(), want, atol=1e-5)
