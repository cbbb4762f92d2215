"""Assemble this rank's text loader and optional decision iterator (reference:
``train/data/loaders.py:29-116``): the dataset / collator pair is chosen from ``--pack`` /
``--multiturn``; the decision stream is a started iterator so its workers spin up before training."""
from dataclasses import dataclass
from typing import Iterator, Optional

from torch.utils.data import DataLoader

from ..cli import parse_int_list
from ..distributed import log, rank, world_size
from . import sft


@dataclass
class TrainingLoaders:
    text: Optional[DataLoader]
    decision: Optional[Iterator]


def _identity(x):
    return x


def build_data_loaders(args, model):
    tok = model.tokenizer
    if args.decision_only and not args.decision_data:
        raise ValueError("--decision_only needs --decision_data")
    if not args.decision_only and not args.dataset:
        raise ValueError("--dataset is required (unless --decision_only)")
    if args.decision_data and args.decision_micro_per_step < 1:
        raise ValueError("--decision_micro_per_step must be >= 1 with --decision_data")
    buckets = parse_int_list(args.length_buckets)
    loader = None
    if not args.decision_only:
        base = sft.JsonlChatDataset(sft.jsonl_paths(args.dataset), rank=rank(), world=world_size(), seed=args.seed)
        if args.pack and args.multiturn:
            dataset = sft.PackedMultiTurnRowDataset(base, tok, bd_size=args.bd_size, max_length=args.max_length,
                                                    max_response_length=args.max_response_length,
                                                    keep_all_reasoning=args.keep_all_reasoning,
                                                    max_segments=args.max_segments,
                                                    image_processor=getattr(model, "image_processor", None),
                                                    max_image_pixels=args.max_image_pixels)
            collate = sft.StreamPackedMultiTurnCollator(tok, bd_size=args.bd_size, max_length=args.max_length,
                                                        length_buckets=buckets)
        elif args.pack:
            dataset = sft.PackedRowDataset(base, tok, max_length=args.max_length,
                                           max_response_length=args.max_response_length,
                                           keep_all_reasoning=args.keep_all_reasoning,
                                           max_segments=args.max_segments, ar_only=args.ar_only)
            collate = sft.StreamPackedCollator(tok, max_length=args.max_length, length_buckets=buckets)
        elif args.multiturn:
            dataset = base
            collate = sft.MultiTurnSftCollator(tok, bd_size=args.bd_size, max_length=args.max_length,
                                               max_response_length=args.max_response_length,
                                               length_buckets=buckets, keep_all_reasoning=args.keep_all_reasoning)
        else:
            dataset = base
            collate = sft.SftCollator(tok, max_length=args.max_length, max_response_length=args.max_response_length,
                                      length_buckets=buckets, keep_all_reasoning=args.keep_all_reasoning)
        loader = DataLoader(dataset, batch_size=args.micro_batch_size, num_workers=args.num_workers,
                            collate_fn=collate, drop_last=True)
        log(f"[data] pack={'on' if args.pack else 'off'} multiturn={'on' if args.multiturn else 'off'} "
            f"collator={type(collate).__name__} batch_size={args.micro_batch_size}")
    decision_iter = None
    if args.decision_data:
        from . import decision as D
        records = D.load_decision_records(args.decision_data.split(","))
        ds = D.DecisionRowDataset(records, tok, rank=rank(), world=world_size(), seed=args.seed,
                                  max_tokens=args.decision_max_tokens, max_state=args.decision_max_state,
                                  max_variant_tokens=args.decision_max_variant_tokens,
                                  p_none_pair=args.decision_p_none_pair)
        decision_iter = iter(DataLoader(ds, batch_size=None, num_workers=min(2, args.num_workers),
                                        collate_fn=_identity))
        log(f"[decision] {len(records)} records | weight {args.decision_loss_weight}")
    return TrainingLoaders(text=loader, decision=decision_iter)
