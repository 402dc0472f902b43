"""Governed text + image prompts: precomputed vision embeddings spliced into the token sequence.

A prompt is an ordered list of parts, each either text token ids or one image's embedding vectors
(hidden-size rows from a CLIP/LLaVA-style encoder that runs outside this package).  Admission is
fail-closed:

* the default policy (``mode=""``) admits text-only prompts; a prompt carrying an image is held in
  quarantine (``MultimodalQuarantined``, with a digest id naming the held images) until the caller
  opts in with ``mode="quarantine"``;
* an admitted image must name an allowed raster media type (png, jpeg, webp, gif, bmp by default;
  ``image/*`` or ``*`` widen it; parameters such as ``; charset=`` are ignored), positive
  dimensions within ``max_image_pixels``, bytes within ``max_image_bytes`` (per image and in
  total), at most ``max_images`` images and ``max_embedding_tokens`` embedding rows in total, and
  every row exactly hidden-size wide;
* any violation denies the whole prompt (``MultimodalDenied``) with the reason in the verdict.

Text rows are the model's (scaled) token embeddings; image rows enter unchanged.  The raw image
bytes never reach the decoder: they only feed the limits and the quarantine digest.

Reference: internal/model/multimodal.go (MultimodalPolicy defaults and validity :200-252,
admitVisionEmbedding :254-295, prepareMultimodalRows :136-198, the quarantine digest :324-343).
"""
from __future__ import annotations

import dataclasses
import hashlib
import struct

import torch

DEFAULT_CONTENT_TYPES = ("image/png", "image/jpeg", "image/webp", "image/gif", "image/bmp")


class MultimodalDenied(ValueError):
    """The prompt is refused; ``verdict`` holds the reason and the accounting so far."""

    def __init__(self, verdict: "Verdict"):
        super().__init__(verdict.reason)
        self.verdict = verdict


class MultimodalQuarantined(PermissionError):
    """The prompt carries images and the policy has not opted in; ``verdict.quarantine_id`` names
    the held images."""

    def __init__(self, verdict: "Verdict"):
        super().__init__(verdict.reason)
        self.verdict = verdict


@dataclasses.dataclass
class Policy:
    mode: str = ""                       # "" (images quarantined) or "quarantine" (images admitted)
    max_images: int = 4
    max_image_bytes: int = 10 << 20
    max_image_pixels: int = 4096 * 4096
    max_embedding_tokens: int = 1024
    allowed_content_types: tuple = DEFAULT_CONTENT_TYPES


@dataclasses.dataclass
class Image:
    media_type: str
    width: int
    height: int
    data: bytes = b""


@dataclasses.dataclass
class VisionEmbedding:
    image: Image
    vectors: torch.Tensor                # [n_rows, hidden]


@dataclasses.dataclass
class Part:
    token_ids: list | None = None
    image: VisionEmbedding | None = None


@dataclasses.dataclass
class Verdict:
    decision: str = "allow"              # allow | quarantine | deny
    mode: str = ""
    reason: str = ""
    quarantine_id: str = ""
    images: int = 0
    image_bytes: int = 0
    embedding_tokens: int = 0


def normalize_media_type(s: str) -> str:
    return s.split(";", 1)[0].strip().lower()


def _deny(v: Verdict, reason: str):
    v.decision, v.reason = "deny", reason
    raise MultimodalDenied(v)


def _check_policy(p: Policy, v: Verdict) -> None:
    if p.mode not in ("", "quarantine"):
        _deny(v, f"unknown multimodal mode {p.mode!r}")
    for name in ("max_images", "max_image_bytes", "max_image_pixels", "max_embedding_tokens"):
        if getattr(p, name) <= 0:
            _deny(v, f"{name} must be positive")
    for ct in p.allowed_content_types:
        c = normalize_media_type(ct)
        if c not in ("*", "image/*") and (not c.startswith("image/") or c == "image/"):
            _deny(v, f"allowed content type {ct!r} must be an image/* media type")


def _admit(e: VisionEmbedding, p: Policy, v: Verdict, hidden: int) -> None:
    v.images += 1
    if v.images > p.max_images:
        _deny(v, "too many images")
    media = normalize_media_type(e.image.media_type)
    if not media.startswith("image/"):
        _deny(v, "media type must be image/*")
    allow = {normalize_media_type(c) for c in p.allowed_content_types}
    if not ({"*", "image/*", media} & allow):
        _deny(v, f"content type {media!r} not on the allow-list")
    if e.image.width <= 0 or e.image.height <= 0:
        _deny(v, "image dimensions must be positive")
    if e.image.width * e.image.height > p.max_image_pixels:
        _deny(v, "image pixel count exceeds limit")
    n = len(e.image.data)
    v.image_bytes += n
    if n > p.max_image_bytes or v.image_bytes > p.max_image_bytes:
        _deny(v, "image bytes exceed limit")
    vec = e.vectors
    if vec.dim() != 2 or vec.shape[0] == 0:
        _deny(v, "image embedding is empty")
    v.embedding_tokens += int(vec.shape[0])
    if v.embedding_tokens > p.max_embedding_tokens:
        _deny(v, "image embedding token count exceeds limit")
    if vec.shape[1] != hidden:
        _deny(v, f"image embedding width {vec.shape[1]}, want {hidden}")


def quarantine_id(parts: list[Part]) -> str:
    """Digest of the held images: media type, size, bytes and embedding rows of each, in order."""
    h = hashlib.sha256()
    for part in parts:
        if part.image is None:
            continue
        im, vec = part.image.image, part.image.vectors.detach().to("cpu", torch.float32).contiguous()
        h.update(f"{normalize_media_type(im.media_type)}|{im.width}|{im.height}|{len(im.data)}|"
                 f"{tuple(vec.shape)}|".encode())
        h.update(im.data)
        h.update(vec.numpy().astype("<f4").tobytes())
        h.update(struct.pack("<q", -1))
    return "vision-sha256:" + h.hexdigest()


def prepare_rows(model, parts: list[Part], policy: Policy | None = None) -> tuple[torch.Tensor, Verdict]:
    """Admit a text + image prompt for ``model`` (a ReferenceModel): (input rows [T, d], verdict)."""
    p = policy or Policy()
    v = Verdict(mode=p.mode)
    _check_policy(p, v)
    if not parts:
        _deny(v, "empty prompt")
    cfg = model.cfg
    rows = []
    for i, part in enumerate(parts):
        has_text, has_image = bool(part.token_ids), part.image is not None
        if has_text == has_image:
            _deny(v, f"part {i} must hold exactly one of token ids or an image embedding")
        if has_text:
            ids = torch.as_tensor(part.token_ids, dtype=torch.long)
            if bool(((ids < 0) | (ids >= cfg.vocab_size)).any()):
                _deny(v, f"token id outside vocab size {cfg.vocab_size}")
            rows.append(model.embed(ids).float())
        else:
            _admit(part.image, p, v, cfg.d_model)
            rows.append(part.image.vectors.to(model.device, torch.float32))
    if v.images and p.mode != "quarantine":
        v.decision, v.reason, v.quarantine_id = ("quarantine", "multimodal input requires explicit quarantine opt-in",
                                                 quarantine_id(parts))
        raise MultimodalQuarantined(v)
    return torch.cat(rows), v


@torch.no_grad()
def forward_multimodal(model, parts: list[Part], policy: Policy | None = None) -> tuple[torch.Tensor, Verdict]:
    """Logits [T, vocab] of an admitted text + image prompt through the reference model."""
    from .reference import rmsnorm
    x, v = prepare_rows(model, parts, policy)
    h = model.forward_band(x, 0, 0, model.cfg.n_layers)
    return model.lm_head(rmsnorm(h, model.t["output_norm.weight"], model.cfg.rms_eps)), v
