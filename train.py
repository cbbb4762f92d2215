#!/usr/bin/env python3
"""Block-diffusion trainer entry point (same CLI as the reference ``train.py``).

    torchrun --nproc_per_node=8 train.py --model_id <hf dir> --dataset <jsonl dir> ...

``--help`` answers without importing torch.
"""
import sys

if any(a in ("-h", "--help") for a in sys.argv[1:]):
    from trida_stack_b200.cli import build_parser
    build_parser().print_help()
    sys.exit(0)

from trida_stack_b200.train import main  # noqa: E402

if __name__ == "__main__":
    main()
