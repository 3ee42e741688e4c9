#!/usr/bin/env python3
"""Puts the reference's own Python code for this path under `oracle/_ref/` (TEST INFRASTRUCTURE, not product code).

The reference implements the folded-expert forward in Python / PyTorch only, so there is nothing to compile: the
"build" is a copy of the three source files the path needs, from the reference checkout where they lie, into a
package skeleton under `oracle/_ref/` (git-ignored, never committed). With it present, `oracle/ref_torch.py` times and
checks against the reference's own `unpack_nvfp4` / `expert_keys` / `reconstruct_group_experts`; without it (no
reference checkout on this machine and no earlier copy) the numpy port in `oracle/folded_moe_oracle.py` is used.

    python oracle/build_ref.py [/path/to/Chronos]
"""
from __future__ import annotations

import os
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
DEST = HERE / "_ref"
FILES = (  # path within the Chronos project
    "chronos_1t/converter/convert_glm53_flash_colab.py",  # pack_nvfp4 / unpack_nvfp4, batched fold / unbind, tail codecs
    "chronos_1t/models/glm53_holo.py",                    # expert_keys, convert_expert_group, reconstruct_group_experts
    "chronos_1t/models/glm53_chronos_spec.py",            # GROUP_SIZE, group_seed_bases
)


def build(reference_root: str | os.PathLike | None = None) -> bool:
    """Returns True when `oracle/_ref` holds the reference files afterwards."""
    root = Path(reference_root or os.environ.get("CHRONOS_REFERENCE", "/root/reference"))
    if not all((root / f).exists() for f in FILES):
        return all((DEST / f).exists() for f in FILES)
    for f in FILES:
        dst = DEST / f
        dst.parent.mkdir(parents=True, exist_ok=True)
        shutil.copyfile(root / f, dst)
    for pkg in ("chronos_1t", "chronos_1t/converter", "chronos_1t/models"):
        (DEST / pkg / "__init__.py").write_text("")  # bare package markers: the reference's own __init__ pulls in unrelated code
    return True


if __name__ == "__main__":
    ok = build(sys.argv[1] if len(sys.argv) > 1 else None)
    print("oracle/_ref:", "ready" if ok else "no reference checkout found")
