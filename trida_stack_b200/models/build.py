"""Build the training model from an HF checkpoint dir (reference: ``train/models/build.py:12-62``).

Routes dense vs hybrid (``config.layer_types`` with linear-attention layers), adds the
``<|mask|>`` token and resizes the vocabulary (unless ``--ar_only``), loads the weights, attaches
the decision head (initialised from ``decision_head.pt`` > ``jev_head.pt`` when present) and casts
to fp32 masters with ``--fp32_master``.
"""
import json
import os

import torch

from ..cli import parse_int_list
from ..distributed import log
from .block_diffusion import BlockDiffusionLM
from .config import ModelConfig
from .decoder import Decoder

MASK_TOKEN = "<|mask|>"


def load_tokenizer(path, trust_remote_code=False):
    try:
        from transformers import AutoTokenizer
        return AutoTokenizer.from_pretrained(path, trust_remote_code=trust_remote_code)
    except Exception as e:  # no tokenizer files: synthetic / weights-only checkpoints
        log(f"[model] no tokenizer in {path} ({type(e).__name__}); token ids must be supplied directly")
        return None


def is_hybrid_dir(path):
    with open(os.path.join(path, "config.json")) as f:
        return ModelConfig.from_hf_dict(json.load(f)).is_hybrid


def load_decoder(path, device, dtype=torch.bfloat16, tokenizer=None, add_mask=True):
    from ..checkpoint import read_hf_weights
    cfg = ModelConfig.from_pretrained(path)
    sd = read_hf_weights(path)
    emb = sd.get("model.embed_tokens.weight", sd.get("model.language_model.embed_tokens.weight"))
    if emb is not None:
        cfg.vocab_size = emb.shape[0]
    dec = Decoder(cfg, dtype=dtype, device=device)
    dec.load_hf_state_dict(sd, strict=True)
    mask_id = None
    if tokenizer is not None:
        if add_mask and MASK_TOKEN not in tokenizer.get_vocab():
            tokenizer.add_special_tokens({"additional_special_tokens": [MASK_TOKEN]})
        if add_mask or len(tokenizer) > cfg.vocab_size:
            dec.resize_vocab(len(tokenizer))
        if MASK_TOKEN in tokenizer.get_vocab():
            mask_id = tokenizer.convert_tokens_to_ids(MASK_TOKEN)
        if tokenizer.pad_token_id is None:
            tokenizer.pad_token = tokenizer.eos_token
    return dec, mask_id


def build_model(args, device=None):
    source = args.resume or args.model_id
    if args.resume:
        from ..checkpoint import verify_manifest
        if verify_manifest(args.resume):
            log(f"[resume] {args.resume}: every file matches its manifest")
        log(f"[resume] loading model weights from {args.resume}")
    device = device or (torch.device("cuda") if torch.cuda.is_available() else torch.device("cpu"))
    tok = load_tokenizer(source, args.trust_remote_code)
    dtype = torch.bfloat16 if device.type == "cuda" else torch.float32
    dec, mask_id = load_decoder(source, device, dtype=dtype, tokenizer=tok, add_mask=not args.ar_only)
    if mask_id is None:
        side = os.path.join(source, "block_diffusion.json")
        mask_id = json.load(open(side))["mask_id"] if os.path.exists(side) else dec.cfg.vocab_size - 1
    common = dict(mask_id=mask_id, pad_id=(tok.pad_token_id if tok is not None else 0), bd_size=args.bd_size,
                  ar_loss_weight=args.ar_loss_weight, loss_weighting=args.loss_weighting,
                  pos_decay_gamma=args.pos_decay_gamma, full_mask=args.full_mask,
                  within_block_causal=args.within_block_causal, mask_pattern=args.mask_pattern,
                  response_buckets=parse_int_list(args.response_buckets), max_length=args.max_length,
                  max_response_length=args.max_response_length, merged_views=args.merged_views,
                  ar_only=args.ar_only, activation_checkpoint=args.activation_checkpoint, tokenizer=tok,
                  activation_offload=getattr(args, "activation_offload", False))
    if dec.cfg.is_hybrid:
        from .hybrid import HybridBlockDiffusionLM
        log(f"[model] hybrid linear-attention decoder -> two-stream objective "
            f"(linear_block_mode={args.linear_block_mode})")
        model = HybridBlockDiffusionLM(dec, linear_block_mode=args.linear_block_mode,
                                       decision_head_dim=args.decision_head_dim if args.decision_data else 0, **common)
    else:
        model = BlockDiffusionLM(dec, **common)
    heads = [os.path.join(source, n) for n in ("decision_head.pt", "jev_head.pt")]
    head_init = next((h for h in heads if os.path.exists(h)), None)
    if getattr(model, "decision_head", None) is not None and head_init:
        saved = torch.load(head_init, map_location="cpu")
        if saved["head_dim"] != args.decision_head_dim:
            raise ValueError(f"{head_init} has head_dim {saved['head_dim']}, --decision_head_dim is {args.decision_head_dim}")
        model.decision_head.load_state_dict(saved["head"])
        log(f"[decision] pointer head initialised from {head_init}")
    if model.is_vl:
        from ..data.images import ImageProcessor
        model.image_processor = ImageProcessor.from_pretrained(source) or ImageProcessor()
        log(f"[model] vision-language checkpoint: frozen vision encoder, trainable projector | "
            f"images capped at {args.max_image_pixels} px")
    if args.fp32_master:
        for p in model.parameters():
            p.data = p.data.float()
    return model.to(device)
