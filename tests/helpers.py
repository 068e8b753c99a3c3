"""Shared test helpers: golden fixture loading and tolerance checks.

Tolerances (from the operator's parity contract):
* outputs O: |got - ref| <= 2e-3 + 1e-2 * |ref| elementwise, in FP32;
* LSE: |got - ref| <= 1e-4 * |ref| + 1e-5;
* sentinel values and block-table indexing: bit-exact.
"""
import glob
import os

import numpy as np
import torch

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
O_ATOL, O_RTOL = 2e-3, 1e-2
LSE_RTOL, LSE_ATOL = 1e-4, 1e-5


def golden_paths():
    return sorted(glob.glob(os.path.join(GOLDEN_DIR, "*.npz")))


def load_golden(path, device="cpu"):
    z = np.load(path)
    dt = getattr(torch, str(z["dtype"]))

    def t16(a, dtype=dt):
        return torch.from_numpy(a.astype(np.int16)).view(dtype).to(device)

    return {
        "name": os.path.basename(path)[:-4],
        "dtype": dt,
        "q": t16(z["q"]),
        "k_cache": t16(z["k_cache"]),
        "v_cache": t16(z["v_cache"]),
        "block_table": torch.from_numpy(z["block_table"]).to(device),
        "seq_len": int(z["seq_len"]),
        "block_size": int(z["block_size"]),
        "num_splits": int(z["num_splits"]),
        "o_ref": t16(z["o_ref"]).float(),
        "o_partial": t16(z["o_partial"], torch.float16).float(),
        "lse_partial": torch.from_numpy(z["lse_partial"]).to(device),
    }


def assert_o_close(got, ref, what=""):
    got = got.float().cpu()
    ref = ref.float().cpu()
    err = (got - ref).abs()
    bound = O_ATOL + O_RTOL * ref.abs()
    bad = err > bound
    assert not torch.isnan(got).any(), f"{what}: NaN in output"
    assert not bad.any(), (f"{what}: {int(bad.sum())} elements out of tolerance, "
                           f"max err {err.max().item():.3e}")


def assert_lse_close(got, ref, what=""):
    got = got.float().cpu()
    ref = ref.float().cpu()
    err = (got - ref).abs()
    bound = LSE_RTOL * ref.abs() + LSE_ATOL
    bad = err > bound
    assert not bad.any(), (f"{what}: {int(bad.sum())} LSE out of tolerance, "
                           f"max err {err.max().item():.3e}")
