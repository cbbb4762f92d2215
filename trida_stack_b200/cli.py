"""Command-line flags of the block-diffusion trainer.

This module imports only ``argparse`` so ``python train.py --help`` answers before torch is
imported.  The flag names, types and defaults are the reference trainer's public interface
(``train/cli.py:9-143`` in trida-stack) so existing launch scripts keep working; the extra flags
at the end (``--mask_pattern``, ``--profile_*``, ``--activation_checkpoint``, ``--comm``) are
B200-specific additions that default to the reference behaviour.
"""
import argparse

def build_parser():
    # allow_abbrev=False: the removed --jev_* spellings must fail (exit code 2), never resolve
    # to a prefix of a current flag.
    p = argparse.ArgumentParser(description="B200 block-diffusion SFT trainer", allow_abbrev=False)
    # ---- model / resume --------------------------------------------------------------------
    p.add_argument("--model_id", default="Qwen/Qwen3.5-4B",
                   help="HF model dir (config.json + safetensors) to convert to block diffusion")
    p.add_argument("--resume", default=None,
                   help="checkpoint dir: loads its weights; also restores optimizer state and "
                        "global_step when train_state/ is present (exact resume), else warm restart")
    p.add_argument("--save_optim_state", action="store_true",
                   help="write the sharded optimizer state next to every checkpoint (exact --resume)")
    p.add_argument("--trust_remote_code", action="store_true")
    p.add_argument("--dataset", default="",
                   help="local dir or file of *.jsonl chat records ({'messages': [...], 'tools': [...]}); "
                        "required unless --decision_only")
    # ---- block-diffusion objective ---------------------------------------------------------
    p.add_argument("--bd_size", type=int, default=32)
    p.add_argument("--max_length", type=int, default=16384)
    p.add_argument("--max_response_length", type=int, default=4096)
    p.add_argument("--length_buckets", default="2048,4096,8192,16384")
    p.add_argument("--response_buckets", default="512,1024,2048,4096")
    p.add_argument("--ar_loss_weight", type=float, default=0.2)
    p.add_argument("--ar_only", action="store_true",
                   help="plain causal-LM SFT (no block-diffusion views, no <|mask|> token)")
    p.add_argument("--loss_weighting", choices=["weighted", "uniform"], default="weighted",
                   help="diffusion CE weighting: 1/gamma ELBO weight normalised to sum 1, or plain mean")
    p.add_argument("--pos_decay_gamma", type=float, default=0.0,
                   help="intra-block positional loss decay exp(-p/gamma); 0 disables")
    p.add_argument("--full_mask", action="store_true",
                   help="mask every response token (gamma=1) with a single noisy view")
    p.add_argument("--linear_block_mode", choices=["causal", "bidirectional"], default="causal",
                   help="hybrid models: gated-delta layers scan causally, or run the two-stream "
                        "block-bidirectional scan")
    p.add_argument("--allow_slow_linear", action="store_true",
                   help="hybrid models: accept the pure-torch gated-delta path when the CUDA "
                        "extension is unavailable")
    p.add_argument("--micro_batch_size", type=int, default=1)
    p.add_argument("--grad_accum", type=int, default=8)
    p.add_argument("--multiturn", action="store_true",
                   help="supervise every assistant turn of a conversation")
    p.add_argument("--keep_all_reasoning", action="store_true",
                   help="keep <think> reasoning on every assistant turn")
    p.add_argument("--pack", action="store_true", help="pack several documents per row (doc-isolated)")
    p.add_argument("--activation_offload", action="store_true",
                   help="with layer checkpointing active, keep each checkpointed layer's input in pinned "
                        "host memory (copied on a side stream) until its backward")
    p.add_argument("--fused_ce", action="store_true",
                   help="accepted for compatibility: the CUDA path always uses the fused linear CE")
    p.add_argument("--fsdp_keep_params", action="store_true",
                   help="keep gathered layer weights resident between forward and backward (no reshard after "
                        "forward)")
    p.add_argument("--shard", choices=["full", "zero2"], default="full",
                   help="full: decoder-layer weights sharded across ranks and gathered per layer (FSDP full "
                        "shard); zero2: replicated weights, sharded gradients and optimizer state")
    p.add_argument("--compile_mlp", action="store_true", help="accepted for compatibility (no-op)")
    p.add_argument("--compile_glue", action="store_true", help="accepted for compatibility (no-op)")
    p.add_argument("--compile_layers", action="store_true", help="accepted for compatibility (no-op)")
    p.add_argument("--merged_views", action="store_true",
                   help="store the shared prompt once for both complementary views (lossless)")
    p.add_argument("--within_block_causal", action="store_true",
                   help="x_t attention inside a block is token-causal instead of bidirectional")
    p.add_argument("--max_segments", type=int, default=0, help="max documents per packed row (0=unlimited)")
    # ---- typed decisions -------------------------------------------------------------------
    p.add_argument("--decision_data", default="",
                   help="comma-separated kev-format JSONL files/dirs for joint pointer-head training")
    p.add_argument("--decision_only", action="store_true",
                   help="train only the typed-decision objective")
    p.add_argument("--decision_loss_weight", type=float, default=1.0)
    p.add_argument("--decision_micro_per_step", type=int, default=1)
    p.add_argument("--decision_max_tokens", type=int, default=32768)
    p.add_argument("--decision_max_variant_tokens", type=int, default=0)
    p.add_argument("--decision_max_state", type=int, default=7552)
    p.add_argument("--decision_p_none_pair", type=float, default=0.25)
    p.add_argument("--decision_head_dim", type=int, default=256)
    p.add_argument("--decision_head_lr_scale", type=float, default=1.0)
    p.add_argument("--projector_lr_scale", type=float, default=0.1)
    p.add_argument("--max_image_pixels", type=int, default=1024 * 1024)
    # ---- optimisation ----------------------------------------------------------------------
    p.add_argument("--max_steps", type=int, default=2000)
    p.add_argument("--start_step", type=int, default=0)
    p.add_argument("--lr", type=float, default=1e-5)
    p.add_argument("--warmup", type=int, default=50)
    p.add_argument("--lr_min_ratio", type=float, default=0.1)
    p.add_argument("--weight_decay", type=float, default=0.0)
    p.add_argument("--adam_beta2", type=float, default=0.95)
    p.add_argument("--fp32_master", action="store_true",
                   help="fp32 master weights and optimizer state (compute stays bf16)")
    p.add_argument("--grad_clip", type=float, default=1.0)
    p.add_argument("--num_workers", type=int, default=2)
    p.add_argument("--seed", type=int, default=42)
    p.add_argument("--log_every", type=int, default=10)
    p.add_argument("--save_every", type=int, default=500)
    p.add_argument("--save_dir", default="checkpoints/hf_block_diffusion")
    p.add_argument("--wandb", action="store_true")
    p.add_argument("--wandb_project", default=None)
    p.add_argument("--run_name", default=None)
    # ---- additions (defaults reproduce the reference behaviour) ----------------------------
    p.add_argument("--mask_pattern", choices=["random", "canvas"], default="random",
                   help="'canvas' = decoder-canvas suffix masks for draft-aligned fine-tuning")
    p.add_argument("--activation_checkpoint", choices=["auto", "none", "layer"], default="auto",
                   help="'auto' keeps activations resident when they fit in HBM, else recomputes "
                        "each layer in backward")
    p.add_argument("--comm", choices=["fused", "nccl"], default="fused",
                   help="multi-GPU parameter/gradient traffic: fused peer-memory kernels or NCCL")
    p.add_argument("--profile_steps", type=int, default=0, help="record this many steps with NVTX/CUDA events")
    p.add_argument("--profile_start", type=int, default=5)
    p.add_argument("--profile_dir", default="profile")
    return p


def parse_int_list(s):
    return tuple(int(x) for x in s.split(",")) if s else None
