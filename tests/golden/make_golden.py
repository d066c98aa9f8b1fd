"""Generate golden vectors by running the reference's own ``run()``.

Run in a container where the reference checkout is present::

    python tests/golden/make_golden.py /path/to/reference

It imports ``flashinfer_baseline.run`` (``flashinfer_baseline.py:5-169``) from
that checkout, feeds it seeded DeepSeek-V3-shaped inputs (H=7168, I=2048,
E=256, E_local=32, the only geometry the reference accepts) and stores the
small tensors plus the reference's bf16 outputs in ``ref_run_v3.npz``.
The 1.4 GB of expert weights are not stored: they are redrawn from the seed by
``gemms_b200.workloads.make_inputs`` and checked against a stored SHA-256.
The GPU box never reads the reference; it only reads this fixture.
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from gemms_b200 import workloads as W  # noqa: E402
from oracle import reference_moe as R  # noqa: E402

SEED = 1
T = 8
OFFSETS = (0, 96, 224)
OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "ref_run_v3.npz")


def golden_shape() -> W.MoeShape:
    return W.CONFIGS["c1"].replace(T=T, shared=False)


def draw():
    """The fixture's inputs: seeded weights for 32 local experts + routing."""
    d = W.make_inputs(golden_shape(), seed=SEED, experts=32)
    logits = R.router_logits(d["x"], d["router_w"])
    hs, hs_scale = R.quantize_1x128(d["x"])
    return d, logits, hs, hs_scale


def weights_digest(d) -> str:
    h = hashlib.sha256()
    for k in ("w13", "w13_scale", "w2", "w2_scale"):
        t = d[k].contiguous()
        h.update(t.view(torch.uint8).numpy().tobytes() if t.dtype == torch.float8_e4m3fn
                 else t.numpy().tobytes())
    return h.hexdigest()


def main(ref_dir: str) -> None:
    sys.path.insert(0, ref_dir)
    import flashinfer_baseline as FB  # the reference oracle, unmodified

    d, logits, hs, hs_scale = draw()
    outs = {}
    for off in OFFSETS:
        y = FB.run(logits, d["router_bias"], hs, hs_scale, d["w13"], d["w13_scale"], d["w2"],
                   d["w2_scale"], off, 2.5)
        outs[f"out_off{off}"] = y.view(torch.int16).numpy()
    np.savez_compressed(
        OUT,
        seed=np.int64(SEED), T=np.int64(T), offsets=np.array(OFFSETS, dtype=np.int64),
        routing_logits=logits.numpy(), routing_bias=d["router_bias"].numpy(),
        hidden_states=hs.view(torch.uint8).numpy(), hidden_states_scale=hs_scale.numpy(),
        weights_sha256=np.array(weights_digest(d)),
        torch_version=np.array(torch.__version__),
        **outs)
    print("wrote", OUT, os.path.getsize(OUT), "bytes")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <reference checkout>")
    main(sys.argv[1])
