"""Shared helpers of the test suite (input generators, oracle adapters)."""
import numpy as np
import torch


def bf16_to_f32(bits):
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def seeded(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


def make_layer_inputs(T, H, I, E, seed=1111, x_std=1.0, w_std=0.02):
    """bf16 x [T,H], router_w [E,H], w1 [E,2I,H], w2 [E,H,I] on the CPU (x ~ N(0, x_std), weights ~ N(0, w_std))."""
    g = seeded(seed)
    x = (torch.randn(T, H, generator=g) * x_std).to(torch.bfloat16)
    rw = (torch.randn(E, H, generator=g) * w_std).to(torch.bfloat16)
    w1 = (torch.randn(E, 2 * I, H, generator=g) * w_std).to(torch.bfloat16)
    w2 = (torch.randn(E, H, I, generator=g) * w_std).to(torch.bfloat16)
    return x, rw, w1, w2


def sf_bytes_of_rows(atoms: np.ndarray, rows: np.ndarray, n_groups: int) -> np.ndarray:
    """Read back the per-row UE8M0 bytes [len(rows), n_groups] from activation SF atoms [MB, KG, 512]."""
    rows = np.asarray(rows, dtype=np.int64)[:, None]
    g = np.arange(n_groups)[None, :]
    byte = 16 * (rows % 32) + 4 * ((rows % 128) // 32) + (g % 4)
    return atoms[rows // 128, g // 4, byte]


def rel_fro(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))
