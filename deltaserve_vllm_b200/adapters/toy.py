"""Toy LoRA adapters for trying the engine: small, well-formed, non-trivial.

    python -m deltaserve_vllm_b200.adapters.toy --model llama3-8b --out adapters
    python -m deltaserve_vllm_b200.adapters.toy --model qwen3-0.6b --out adapters --count 32 --name topic

Each adapter is trained by this engine itself (finetuning-only steps, no
inference load) for a couple of epochs on a generated topic corpus, then
written as a PEFT directory ``<out>/<name>`` plus an identical
``<out>/<name>-ft`` to use as the finetuning target, and the corpus as
``<out>/<name>/data.txt`` (a ``data_path`` for finetuning jobs and for the
adapter-routing index). With ``--count N`` the adapters get N different
topics, so routing has something to tell apart.

Same role as the reference's toy adapter builders
(``scripts/toy_adapters.py``, ``scripts/init_adapters_llama3.py``): those
train rank-16 q/k/v/o adapters with a separate HF Trainer run; here the
engine's own LoRA backward does the training.
"""

from __future__ import annotations

import argparse
import json
import os
import random
import shutil

_TOPICS = {
    "cooking": ("simmer", "garlic", "saute", "broth", "oven", "knead", "dough", "spice", "roast", "whisk"),
    "astronomy": ("nebula", "orbit", "galaxy", "comet", "parallax", "quasar", "redshift", "eclipse", "pulsar", "lunar"),
    "law": ("statute", "plaintiff", "appeal", "tort", "verdict", "clause", "counsel", "precedent", "liability", "writ"),
    "sailing": ("jib", "tack", "keel", "mainsail", "leeward", "starboard", "mooring", "gust", "hull", "rigging"),
    "chess": ("gambit", "rook", "castle", "endgame", "pawn", "bishop", "checkmate", "opening", "fork", "tempo"),
    "biology": ("enzyme", "cell", "protein", "mitosis", "gene", "membrane", "ribosome", "allele", "tissue", "neuron"),
    "music": ("chord", "tempo", "octave", "melody", "cadence", "timbre", "rhythm", "sonata", "harmony", "scale"),
    "finance": ("bond", "yield", "equity", "dividend", "ledger", "hedge", "margin", "audit", "asset", "liquidity"),
}
_FRAMES = ("Explain how {a} relates to {b}.", "A short note on {a}, {b} and {c}.",
           "Why does {a} matter when working with {b}?", "Describe {a} in one sentence, then {b}.",
           "List three facts about {a}: {b}, {c}, and more.")


def topic_corpus(topic_id: int, n: int = 96, seed: int = 0) -> list[str]:
    """``n`` short lines about one generated topic (topics beyond the built-in
    list reuse their word lists with a distinct suffix)."""
    names = sorted(_TOPICS)
    base = names[topic_id % len(names)]
    words = [w + (f"-{topic_id // len(names)}" if topic_id >= len(names) else "") for w in _TOPICS[base]]
    rng = random.Random(seed * 7919 + topic_id)
    out = []
    for _ in range(n):
        a, b, c = rng.sample(words, 3)
        out.append(rng.choice(_FRAMES).format(a=a, b=b, c=c) + f" ({base})")
    return out


def train_toy_adapter(model: str, out_dir: str, name: str, topic_id: int, rank: int = 16, alpha: float = 32.0,
                      targets=("q", "k", "v", "o"), epochs: int = 2, device: str | None = None,
                      seed: int = 0, lr: float = 2e-4) -> str:
    """Train one toy adapter with the engine and write ``<out_dir>/<name>``
    (+ ``-ft`` copy and ``data.txt``). Returns the adapter directory."""
    from ..config import EngineConfig, FinetuneConfig
    from ..engine.ft.store import FinetuningStore
    from ..engine.llm_engine import CoServingEngine
    from ..models.configs import resolve_arch
    from ..utils.tokenizer import load_tokenizer

    arch = resolve_arch(model)
    tok = load_tokenizer(model if os.path.isdir(model) else None, arch.vocab)
    lines = topic_corpus(topic_id, seed=seed)
    cap = 256
    ecfg = EngineConfig(model=model, device=device, max_model_len=1024, block_size=16,
                        max_num_batched_tokens=2048, max_loras=2, max_lora_rank=rank, seed=seed)
    fcfg = FinetuneConfig(enable_finetuning=True, max_saved_finetuning_tokens=cap, learning_rate=lr,
                          num_epochs=epochs, ft_target_modules=list(targets), profile_on_launch=False)
    store = FinetuningStore(None, None, None, total_epochs=epochs, max_saved_finetuning_tokens=cap)
    store.add_samples((tok.encode(t), t) for t in lines)
    from . import peft_io
    from ..models.lora import random_adapter
    init = random_adapter(arch, rank, seed=seed + 17 * topic_id, targets=tuple(targets), b_std=0.0)
    eng = CoServingEngine(ecfg, fcfg, arch=arch, tokenizer=tok, ft_store=store, ft_adapter=(init, rank, alpha))
    eng.run_until_idle(max_steps=100000)
    path = os.path.join(out_dir, name)
    eng.save_adapter(path, save_id=name)
    # the saved config lists every projection the masters hold; keep the trained subset
    cfg = dict(peft_io.default_adapter_config(rank, alpha, targets, model),
               base_model_name_or_path=model)
    with open(os.path.join(path, peft_io.CONFIG_FILE), "w") as f:
        json.dump(cfg, f, indent=2)
    with open(os.path.join(path, "data.txt"), "w") as f:
        f.write("\n".join(lines) + "\n")
    ft = path + "-ft"
    if os.path.exists(ft):
        shutil.rmtree(ft)
    shutil.copytree(path, ft)
    eng.close()
    return path


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--model", required=True, help="preset name or HF model directory")
    ap.add_argument("--out", default="adapters")
    ap.add_argument("--name", default="toy")
    ap.add_argument("--count", type=int, default=1, help="number of adapters (distinct topics)")
    ap.add_argument("--rank", type=int, default=16)
    ap.add_argument("--alpha", type=float, default=32.0)
    ap.add_argument("--targets", default="q,k,v,o", help="comma-separated subset of q,k,v,o,gate,up,down")
    ap.add_argument("--epochs", type=int, default=2)
    ap.add_argument("--device", default=None)
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)
    os.makedirs(a.out, exist_ok=True)
    targets = tuple(t.strip() for t in a.targets.split(",") if t.strip())
    for i in range(a.count):
        name = a.name if a.count == 1 else f"{a.name}-{i:02d}"
        p = train_toy_adapter(a.model, a.out, name, i, a.rank, a.alpha, targets, a.epochs, a.device, a.seed)
        print(p, flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
