"""Time the decode matvec over one weight tensor of a synthetic BASELINE-shape model.

    python -m dotllm_b200.profile CONFIG TENSOR [BATCH [ITERS]]
    e.g. python -m dotllm_b200.profile llama1b-shape token_embd.weight 1 3

TENSOR may name every layer's copy with `blk.*.` (the launches then cycle through the layers,
so repeated launches do not hit L2).  Prints the average device time per launch (CUDA events
around a CUDA graph of ITERS passes) and the bandwidth of the quantised bytes.  This is the
command the ncu summaries under profiles/ run under `ncu -k regex:gemv_mma_kernel`.
"""
from __future__ import annotations

import sys

from . import synth
from .engine import CudaModel


def main(argv=None) -> None:
    argv = sys.argv[1:] if argv is None else argv
    if len(argv) < 2:
        raise SystemExit(__doc__)
    name, tensor = argv[0], argv[1]
    batch = int(argv[2]) if len(argv) > 2 else 1
    iters = int(argv[3]) if len(argv) > 3 else 10
    m = CudaModel.load(synth.build_model(synth.get(name)))
    try:
        ms, nb = m.profile_matvec(tensor, batch, iters)
    finally:
        m.close()
    print(f"{name} {tensor} rows={batch}: {ms * 1000:.2f} us per launch, {nb / 1e6:.2f} MB, "
          f"{nb / ms / 1e6:.1f} GB/s", flush=True)


if __name__ == "__main__":
    main()
