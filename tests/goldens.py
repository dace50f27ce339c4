"""Loader for the committed golden fixtures (outputs of the reference, see tests/golden/gen_golden.py)."""
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


def plan_of(g: dict) -> dict:
    keys = ("src_y", "src_v", "src_t", "src_id", "cell_start", "anc_x", "anc_t", "anc_cell", "anc_id", "slice_c")
    p = {k: g[k] for k in keys}
    p.update(S=int(g["S"]), GH=int(g["GH"]), GW=int(g["GW"]))
    return p


def sort_within_cells(p: dict):
    """(src_id, y, v, t) re-ordered by (cell, src_id): the reference's argsort is unstable within a cell."""
    cs = p["cell_start"]
    cell_of = np.repeat(np.arange(cs.shape[0] - 1), np.diff(cs))
    order = np.lexsort((p["src_id"], cell_of))
    return p["src_id"][order], p["src_y"][order], p["src_v"][order], p["src_t"][order]
