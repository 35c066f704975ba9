"""Loader for the golden vectors in tests/golden (see make_golden.py there)."""
import glob
import os

import numpy as np
import torch

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
_DT = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}


def _tensor(arr, dtype):
    if dtype in (torch.float16, torch.bfloat16):
        return torch.from_numpy(arr.view(np.int16).copy()).view(dtype)
    return torch.from_numpy(arr.copy())


def cases():
    return sorted(os.path.splitext(os.path.basename(p))[0] for p in glob.glob(os.path.join(GOLDEN_DIR, "*.npz")))


def load(name):
    z = np.load(os.path.join(GOLDEN_DIR, name + ".npz"))
    dt = _DT[str(z["dtype"])]
    return {
        "q": _tensor(z["q"], dt), "k": _tensor(z["k"], dt), "v": _tensor(z["v"], dt), "dtype": dt,
        "causal": bool(z["causal"]), "out_ref": _tensor(z["out_ref"], dt),
        "out_ref_fp32": torch.from_numpy(z["out_ref_fp32"].copy()),
    }
