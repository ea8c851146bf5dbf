"""Record the reference kernels' own outputs as golden fixtures (GPU run).

Runs thebigblender/FlashLite's forward_flash2 and forward_naive (built from
its sources for sm_100a by oracle/build_ref.py) on the inputs of every
tests/golden/golden_*.npz and writes ref_<name>.npz (fp16 outputs) to the
directory given as argv[1] (default: this directory). The CPU test
tests/test_reference_golden.py then pins the oracle on these outputs.

Run on a B200 from the repository root:
    python tests/golden/make_ref_golden.py [out_dir]
"""
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from oracle import build_ref  # noqa: E402


def main():
    out_dir = Path(sys.argv[1]) if len(sys.argv) > 1 else Path(__file__).parent
    out_dir.mkdir(parents=True, exist_ok=True)
    mod = build_ref.load()
    if mod is None:
        raise SystemExit("oracle/_ref not built")
    for g in sorted(Path(__file__).parent.glob("golden_*.npz")):
        d = np.load(g)
        q, k, v = (torch.from_numpy(d[n]).cuda() for n in ("q", "k", "v"))
        sm, causal = float(d["sm_scale"]), bool(d["is_causal"])
        o_f2 = mod.forward_flash2(q, k, v, sm, causal).cpu().numpy()
        o_nv = mod.forward_naive(q, k, v, sm, causal).cpu().numpy()
        name = g.stem.replace("golden_", "ref_")
        np.savez_compressed(out_dir / f"{name}.npz", flash2=o_f2, naive=o_nv,
                            device=np.str_(torch.cuda.get_device_name(0)))
        print("wrote", name)


if __name__ == "__main__":
    main()
