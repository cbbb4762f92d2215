"""Images for vision-language (Qwen3.5 VL) SFT: references, loading, preprocessing, placeholder
expansion and 3-D RoPE positions.

Contract (``train/data/text_sft_data.py:69-182``):

* image parts are ``{"type": "image", "image": ref}`` / ``{"image": ref}`` / ``{"image_url": ref or
  {"url": ref}}`` inside a message's ``content`` list, in the order the chat template emits its
  ``<|image_pad|>`` placeholders; refs are paths (relative ones resolve against the record's
  ``image_root``), ``file://`` paths or base64 ``data:`` URIs; video parts are rejected;
* each image is resized so both sides are multiples of ``patch * merge`` and its area stays within
  ``[min_pixels, max_pixels]`` (aspect ratio kept as closely as possible), bicubic, scaled to [0, 1]
  and normalised by the checkpoint's mean / std, duplicated along time to the temporal patch size,
  and cut into ``[C * T * p * p]`` patches ordered ``(t, block_row, block_col, row, col)`` over
  ``merge x merge`` blocks -- the layout the vision tower's patch embedding and merger read;
* the template's single placeholder per image becomes one ``<|image_pad|>`` per merged patch;
* text advances the (t, h, w) positions together, an image's tokens take ``start + (0, row, col)``
  over its merged grid and the next position is ``start + max(h, w) / merge``.

The implementation is this package's own (PIL + numpy), with no transformers image processor.
"""
import base64
import io
import json
import math
import os

import numpy as np
import torch

IMAGE_PAD = "<|image_pad|>"


def image_pad_id(tokenizer):
    """``<|image_pad|>`` id, or None when the tokenizer has no such token (cached on the tokenizer)."""
    pid = getattr(tokenizer, "_trida_image_pad_id", -1)
    if pid == -1:
        vocab = tokenizer.get_vocab()
        pid = vocab.get(IMAGE_PAD)
        try:
            tokenizer._trida_image_pad_id = pid
        except AttributeError:
            pass
    return pid


def is_image_part(part):
    return isinstance(part, dict) and ("image" in part or "image_url" in part or part.get("type") == "image")


def image_refs(messages):
    refs = []
    for m in messages:
        content = m.get("content")
        if not isinstance(content, list):
            continue
        for part in content:
            if is_image_part(part):
                ref = part.get("image") or part.get("image_url")
                refs.append(ref.get("url") if isinstance(ref, dict) else ref)
            elif isinstance(part, dict) and ("video" in part or part.get("type") == "video"):
                raise ValueError("video content is not supported")
    return refs


def load_image(ref, image_root=None):
    from PIL import Image
    if ref.startswith("data:"):
        img = Image.open(io.BytesIO(base64.b64decode(ref.split(",", 1)[1])))
    else:
        path = ref[len("file://"):] if ref.startswith("file://") else ref
        if image_root and not os.path.isabs(path):
            path = os.path.join(image_root, path)
        img = Image.open(path)
    return img.convert("RGB")


def fit_size(height, width, factor, min_pixels, max_pixels, frames=1, upscale_small=False):
    """(h, w) multiples of ``factor`` nearest the input, rescaled so ``frames * h * w`` lies in
    ``[min_pixels, max_pixels]``.  GLM-style processors count the temporal frames in the pixel
    budget (``frames`` = temporal patch size) and first scale up images with a side below
    ``factor`` (``upscale_small``)."""
    if upscale_small and (height < factor or width < factor):
        sc = max(factor / height, factor / width)
        height, width = int(height * sc), int(width * sc)
    if max(height, width) / min(height, width) > 200:
        raise ValueError(f"image aspect ratio {max(height, width) / min(height, width):.1f} exceeds 200")
    h = round(height / factor) * factor
    w = round(width / factor) * factor
    if frames * h * w > max_pixels:
        s = math.sqrt(frames * height * width / max_pixels)
        h = max(factor, math.floor(height / s / factor) * factor)
        w = max(factor, math.floor(width / s / factor) * factor)
    elif frames * h * w < min_pixels:
        s = math.sqrt(min_pixels / (frames * height * width))
        h = math.ceil(height * s / factor) * factor
        w = math.ceil(width * s / factor) * factor
    return h, w


class ImageProcessor:
    """Qwen-VL style patch preprocessing configured from a checkpoint's ``preprocessor_config.json``."""

    def __init__(self, patch_size=16, temporal_patch_size=2, merge_size=2, min_pixels=56 * 56,
                 max_pixels=28 * 28 * 1280, image_mean=(0.5, 0.5, 0.5), image_std=(0.5, 0.5, 0.5),
                 rescale_factor=1.0 / 255, raw=None, glm=False):
        self.patch_size, self.temporal_patch_size, self.merge_size = patch_size, temporal_patch_size, merge_size
        self.min_pixels, self.max_pixels = min_pixels, max_pixels
        self.image_mean = np.asarray(image_mean, dtype=np.float32)
        self.image_std = np.asarray(image_std, dtype=np.float32)
        self.rescale_factor = rescale_factor
        self.raw = raw
        self.glm = glm              # GLM-V resize rule (frames in the pixel budget, small images scaled up)

    @classmethod
    def from_dict(cls, d, glm=None):
        if isinstance(d.get("image_processor"), dict):      # processor_config.json nests it
            d = d["image_processor"]
        if glm is None:
            glm = "glm" in str(d.get("image_processor_type", "")).lower()
        size = d.get("size") or {}
        return cls(patch_size=d.get("patch_size", 16), temporal_patch_size=d.get("temporal_patch_size", 2),
                   merge_size=d.get("merge_size", 2),
                   min_pixels=d.get("min_pixels") or size.get("shortest_edge") or 56 * 56,
                   max_pixels=d.get("max_pixels") or size.get("longest_edge") or 28 * 28 * 1280,
                   image_mean=d.get("image_mean", (0.5, 0.5, 0.5)), image_std=d.get("image_std", (0.5, 0.5, 0.5)),
                   rescale_factor=d.get("rescale_factor", 1.0 / 255), raw=dict(d), glm=glm)

    @classmethod
    def from_pretrained(cls, path, glm=None):
        for name in ("preprocessor_config.json", "processor_config.json"):
            f = os.path.join(path, name)
            if os.path.exists(f):
                with open(f) as fh:
                    return cls.from_dict(json.load(fh), glm=glm)
        return None

    def to_dict(self):
        d = dict(self.raw or {})
        d.update({"patch_size": self.patch_size, "temporal_patch_size": self.temporal_patch_size,
                  "merge_size": self.merge_size, "image_mean": self.image_mean.tolist(),
                  "image_std": self.image_std.tolist(), "rescale_factor": self.rescale_factor,
                  "size": {"shortest_edge": self.min_pixels, "longest_edge": self.max_pixels}})
        d.setdefault("image_processor_type", "Qwen2VLImageProcessor")
        return d

    def save_pretrained(self, path):
        with open(os.path.join(path, "preprocessor_config.json"), "w") as f:
            json.dump(self.to_dict(), f, indent=2)

    def patches(self, img, max_pixels=None):
        """One PIL image -> (patches [t*h*w, C*T*p*p] float32, (t, h, w))."""
        from PIL import Image
        p, m, tp = self.patch_size, self.merge_size, self.temporal_patch_size
        cap = self.max_pixels if max_pixels is None else min(self.max_pixels, max_pixels)
        W0, H0 = img.size
        if self.glm:
            h, w = fit_size(H0, W0, p * m, self.min_pixels, cap, frames=tp, upscale_small=True)
        else:
            h, w = fit_size(H0, W0, p * m, self.min_pixels, cap)
        if (h, w) != (H0, W0):
            img = img.resize((w, h), Image.BICUBIC)
        a = np.asarray(img, dtype=np.float32) * self.rescale_factor
        a = ((a - self.image_mean) / self.image_std).transpose(2, 0, 1)       # [C, h, w]
        C = a.shape[0]
        frames = np.repeat(a[None], tp, axis=0)                               # one image -> tp frames
        gt, gh, gw = 1, h // p, w // p
        x = frames.reshape(gt, tp, C, gh // m, m, p, gw // m, m, p)
        x = x.transpose(0, 3, 6, 4, 7, 2, 1, 5, 8)                            # t, bh, bw, r, c | C, T, p, p
        return x.reshape(gt * gh * gw, C * tp * p * p), (gt, gh, gw)

    def __call__(self, images, max_pixels=None):
        outs, grids = [], []
        for img in images:
            pv, g = self.patches(img, max_pixels)
            outs.append(pv)
            grids.append(g)
        return torch.from_numpy(np.concatenate(outs)), torch.tensor(grids, dtype=torch.long)


def process_images(processor, refs, image_root=None, max_image_pixels=1024 * 1024):
    """(pixel_values [P, C*T*p*p], image_grid_thw [N, 3], merged tokens per image)."""
    pv, grid = processor([load_image(r, image_root) for r in refs], max_image_pixels)
    counts = (grid.prod(-1) // processor.merge_size ** 2).tolist()
    return pv, grid, counts


def expand_image_pads(ids, pad_id, counts):
    """One ``pad_id`` per merged patch instead of one per image; a prefix render holding only the
    first images expands identically (counts are consumed in order)."""
    out, k = [], 0
    for t in ids:
        if t == pad_id:
            out.extend([pad_id] * counts[k])
            k += 1
        else:
            out.append(t)
    return out


def mrope_position_ids(input_ids, image_grid_thw, image_token_id, merge=2):
    """3-D (t, h, w) RoPE positions [3, T] of one document."""
    ids = torch.as_tensor(input_ids)
    T = ids.shape[0]
    img = (ids == image_token_id).tolist()
    pos = torch.empty(3, T, dtype=torch.long)
    grids = iter(image_grid_thw.tolist() if image_grid_thw is not None else [])
    cur, i = 0, 0
    while i < T:
        j = i
        while j < T and img[j] == img[i]:
            j += 1
        n = j - i
        if not img[i]:
            pos[:, i:j] = torch.arange(cur, cur + n)
            cur += n
        else:
            _, gh, gw = next(grids)
            h, w = gh // merge, gw // merge
            if n != h * w:
                raise ValueError(f"image span of {n} tokens does not match its {h}x{w} merged grid")
            pos[0, i:j] = cur
            pos[1, i:j] = cur + torch.arange(h).repeat_interleave(w)
            pos[2, i:j] = cur + torch.arange(w).repeat(h)
            cur += max(gh, gw) // merge
        i = j
    return pos
