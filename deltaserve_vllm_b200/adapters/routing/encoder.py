"""Sentence encoders for routing and indexing.

* :class:`SentenceEncoder` — a local Hugging Face encoder directory (the e5
  family by default): prefix, truncate, mean-pool the last hidden state over
  the attention mask, L2-normalise (as the reference's
  ``deltaserve-plugin/deltaserve/adapter_routing/encoder.py:70-110``). Runs on
  the serving GPU when one is present; the routed requests of a step are
  encoded in one batch.
* :class:`HashingEncoder` — an offline encoder for hosts without encoder
  weights: signed feature hashing of lower-cased word unigrams and bigrams
  (sub-linear term frequency) into a fixed dimension, L2-normalised.
  Deterministic across processes (keyed BLAKE2b, not Python's salted hash).

``make_encoder`` picks the first when ``adapter_routing.encoder`` is a local
directory and the second otherwise (no network here to fetch weights).
"""

from __future__ import annotations

import hashlib
import os
import re

import numpy as np

from ... import dprint

_WORD = re.compile(r"\w+", re.UNICODE)


class HashingEncoder:
    name = "hashing-1024"

    def __init__(self, dim: int = 1024, prefix: str = "", max_tokens: int = 512):
        self.dim, self.prefix, self.max_tokens = int(dim), prefix, int(max_tokens)
        self._cache: dict[str, tuple[int, float]] = {}
        self.loaded = True

    def _slot(self, feat: str) -> tuple[int, float]:
        hit = self._cache.get(feat)
        if hit is None:
            h = int.from_bytes(hashlib.blake2b(feat.encode("utf-8"), digest_size=8).digest(), "little")
            hit = (h % self.dim, 1.0 if (h >> 63) & 1 else -1.0)
            if len(self._cache) < 1 << 20:
                self._cache[feat] = hit
        return hit

    def encode(self, texts: list[str], batch_size: int = 0) -> np.ndarray:
        out = np.zeros((len(texts), self.dim), np.float32)
        for r, t in enumerate(texts):
            words = _WORD.findall(t.lower())[: self.max_tokens]
            feats: dict[str, int] = {}
            for i, w in enumerate(words):
                feats[w] = feats.get(w, 0) + 1
                if i:
                    bg = words[i - 1] + " " + w
                    feats[bg] = feats.get(bg, 0) + 1
            for f, n in feats.items():
                j, sgn = self._slot(f)
                out[r, j] += sgn * (1.0 + np.log(n))
        n = np.linalg.norm(out, axis=1, keepdims=True)
        return out / np.where(n == 0, 1.0, n)

    def unload(self) -> None:
        pass


class SentenceEncoder:
    def __init__(self, path: str, prefix: str = "query: ", max_tokens: int = 512, device: str = "cpu"):
        self.path, self.prefix, self.max_tokens, self.device = path, prefix, int(max_tokens), device
        self.name = os.path.basename(os.path.normpath(path))
        self._tok = self._model = None

    @property
    def loaded(self) -> bool:
        return self._model is not None

    def load(self) -> None:
        if self._model is not None:
            return
        import torch
        from transformers import AutoModel, AutoTokenizer
        self._tok = AutoTokenizer.from_pretrained(self.path, local_files_only=True)
        dtype = torch.bfloat16 if str(self.device).startswith("cuda") else torch.float32
        self._model = AutoModel.from_pretrained(self.path, local_files_only=True,
                                                torch_dtype=dtype).to(self.device).eval()

    def unload(self) -> None:
        self._tok = self._model = None

    # ------------------------------------------------ sharing with a child process
    def shared_state(self) -> tuple[dict, dict]:
        """(model config, every parameter and buffer by name): what a child
        process needs to run this encoder on the SAME tensors. Sent over a
        ``torch.multiprocessing`` pipe, CUDA tensors travel as IPC handles
        (the child maps this process's device memory) and CPU tensors move
        to shared memory; the caller keeps this encoder loaded for as long as
        the child uses them."""
        self.load()
        state = {n: p.detach() for n, p in self._model.named_parameters()}
        state.update({n: b for n, b in self._model.named_buffers()})
        return self._model.config.to_dict(), state

    @classmethod
    def from_shared(cls, path: str, prefix: str, max_tokens: int, device: str, config: dict,
                    state: dict) -> "SentenceEncoder":
        """An encoder whose module is built around ``state``'s tensors (from
        :meth:`shared_state` of another process): the architecture comes from
        ``config`` on the meta device, so no weight is allocated or read here;
        the tokenizer is read from ``path``."""
        import torch
        from transformers import AutoConfig, AutoModel, AutoTokenizer
        enc = cls(path, prefix, max_tokens, device)
        enc._tok = AutoTokenizer.from_pretrained(path, local_files_only=True)
        with torch.device("meta"):
            model = AutoModel.from_config(AutoConfig.for_model(**config))
        named = dict(model.named_parameters())
        named.update(dict(model.named_buffers()))
        missing = sorted(set(named) - set(state))
        if missing:
            raise RuntimeError(f"shared encoder state lacks {missing[:4]}")
        for name, t in state.items():
            owner, _, leaf = name.rpartition(".")
            mod = model.get_submodule(owner) if owner else model
            if leaf in mod._parameters:
                mod._parameters[leaf] = torch.nn.Parameter(t, requires_grad=False)
            elif leaf in mod._buffers:
                mod._buffers[leaf] = t
        enc._model = model.eval()
        return enc

    def layers(self):
        """The encoder's layer stack (its longest ``ModuleList``), or []."""
        import torch
        self.load()
        best = []
        for m in self._model.modules():
            if isinstance(m, torch.nn.ModuleList) and len(m) > len(best):
                best = m
        return list(best)

    def encode(self, texts: list[str], batch_size: int = 16) -> np.ndarray:
        import torch
        self.load()
        chunks = []
        with torch.inference_mode():
            for i in range(0, len(texts), batch_size):
                enc = self._tok([self.prefix + t for t in texts[i:i + batch_size]], padding=True,
                                truncation=True, max_length=self.max_tokens,
                                return_tensors="pt").to(self.device)
                h = self._model(**enc).last_hidden_state.float()
                m = enc["attention_mask"].unsqueeze(-1).float()
                pooled = (h * m).sum(1) / m.sum(1).clamp(min=1.0)
                chunks.append(torch.nn.functional.normalize(pooled, dim=-1).cpu().numpy())
        return np.concatenate(chunks) if chunks else np.zeros((0, 0), np.float32)


def make_encoder(cfg, device: str = "cpu"):
    """The encoder named by an :class:`AdapterRoutingConfig`."""
    if cfg.encoder and os.path.isdir(cfg.encoder):
        dev = device
        if cfg.router_device not in ("auto", None, ""):
            dev = cfg.router_device
        if cfg.router_gpu is not None and str(dev).startswith("cuda"):
            dev = f"cuda:{int(cfg.router_gpu)}"
        return SentenceEncoder(cfg.encoder, cfg.encoder_query_prefix, cfg.encoder_max_tokens, dev)
    dprint(f"[router] encoder '{cfg.encoder}' is not a local directory; using the offline "
           f"hashing encoder")
    return HashingEncoder(prefix=cfg.encoder_query_prefix, max_tokens=cfg.encoder_max_tokens)


def encoder_identity(enc) -> str:
    return getattr(enc, "name", type(enc).__name__)
