import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN_DIR = Path(__file__).resolve().parent / "golden"
GOLDEN_CASES = ("k4_h256_i128", "k8_h384_i128")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (run on the B200 box)")


def load_golden(name: str) -> dict:
    z = np.load(GOLDEN_DIR / f"{name}.npz")
    return {k: z[k] for k in z.files}


def golden_groups(gold: dict) -> list[dict]:
    """Slot tensor dicts (on-disk suffix -> array) of a golden case."""
    h, i, e, k = (int(v) for v in gold["meta"][:4])
    groups = []
    for g in range(e // k):
        pre = f"g{g}."
        groups.append({kk[len(pre):]: v for kk, v in gold.items() if kk.startswith(pre)})
    return groups


@pytest.fixture(params=GOLDEN_CASES)
def golden(request):
    return load_golden(request.param)


ROUTER_CASE = "router_e288_h4096"
NEAR_TIE = 4e-6  # fp32 summation error of a 4096-term logit of magnitude ~1: two orders of summation may disagree below this


def router_case():
    """The router-only golden case at the benchmark's shape. The inputs are regenerated from the stored seed with
    torch's CPU generator exactly as tests/golden/make_golden.py draws them; the file holds the reference's outputs."""
    import torch

    gold = load_golden(ROUTER_CASE)
    e, h, t, k, seed = (int(v) for v in gold["meta"])
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(t, h, generator=gen).to(torch.bfloat16).float()
    router_w = torch.randn(e, h, generator=gen) * 0.02
    e_bias = torch.randn(e, generator=gen) * 0.05
    return gold, x.numpy(), router_w.numpy(), e_bias.numpy(), k


def router_choice_scores(logits: np.ndarray, flavour: str, e_bias: np.ndarray) -> np.ndarray:
    """The scores each flavour ranks by, from the reference's own logits (float64 evaluation of the expressions)."""
    lg = logits.astype(np.float64)
    if flavour == "softmax":
        return lg
    if flavour == "sigmoid":
        return 1.0 / (1.0 + np.exp(-lg)) + e_bias[None, :]
    return np.sqrt(np.where(lg > 20.0, lg, np.log1p(np.exp(lg)))) + e_bias[None, :]


def compare_router_ids(ids: np.ndarray, ref_ids: np.ndarray, choice: np.ndarray, k: int, tol: float = NEAR_TIE) -> dict:
    """Counts tokens whose ids differ from the reference's and, separately, tokens that hold a near-tie: two of their
    k+1 best choice scores closer than `tol`, so two correct fp32 evaluations may order them differently. A mismatch
    on a token without a near-tie is a true mismatch."""
    top = -np.sort(-choice, axis=1)[:, :k + 1]
    near = (np.abs(np.diff(top, axis=1)) < tol).any(axis=1)
    differ = (ids.astype(np.int64) != ref_ids.astype(np.int64)).any(axis=1)
    return {"tokens": int(ids.shape[0]), "near_tie_tokens": int(near.sum()), "mismatch_tokens": int(differ.sum()),
            "true_mismatch_tokens": int((differ & ~near).sum())}
