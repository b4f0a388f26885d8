"""BLiMP minimal pairs (Warstadt et al. 2020, arXiv:1912.00582) for candidate caption LMs (reference blimp_eval.py): a
model passes a pair when the grammatical sentence gets the higher total log-probability; accuracy per paradigm and
overall (chance = 50 %).

  python blimp_eval.py models/slayer149 hf:models/poziomka --data blimp/ --tokenizer tok.json --out blimp.json
  python blimp_eval.py models/slayer149 --data blimp/ --limit 100       # 100 pairs per paradigm

--data: a local copy of the dataset, one file per paradigm (*.jsonl or *.parquet with sentence_good / sentence_bad
columns; the paradigm is the file name or its UID column). Models: a Slayer GPT directory (config.json +
model.safetensors, models/slayer.py), or "hf:<dir>" for a local transformers causal LM. Each sentence gets a
beginning-of-text token in front, so its first word is scored too. Sentences are scored in batches, padded, with
the log-probability of every real token summed.

  python blimp_eval.py hf:models/poziomka --data blimp/ --tokenizer tok.json --set num_experts_per_tok=16 --quant int8

--set KEY=VALUE overrides (JSON values) go into a transformers model's config (e.g. fewer active experts of an MoE);
--quant int8 runs its mixture-of-experts blocks as stacked int8 experts (models/moe_infer.py). Rows that carry a
linguistics_term column are also summarised per phenomenon.
"""
import argparse
import glob
import json
import os
import time

import torch
import torch.nn.functional as F


def load_pairs(data, limit=0, phenomena=None):
    """[(paradigm, good, bad)] from the files under ``data``; ``phenomena`` (a dict), when given, is filled with
    paradigm -> linguistics_term for the rows that carry one."""
    out = []
    for f in sorted(glob.glob(os.path.join(data, "*.jsonl")) + glob.glob(os.path.join(data, "*.parquet"))):
        name = os.path.basename(f).rsplit(".", 1)[0]
        if f.endswith(".jsonl"):
            rows = [json.loads(line) for line in open(f) if line.strip()]
        else:
            import pyarrow.parquet as pq
            rows = pq.read_table(f).to_pylist()
        if limit:
            rows = rows[:limit]
        out += [(r.get("UID", name), r["sentence_good"], r["sentence_bad"]) for r in rows]
        if phenomena is not None:
            phenomena.update({r.get("UID", name): r["linguistics_term"] for r in rows if r.get("linguistics_term")})
    return out


class Scorer:
    """Summed token log-probabilities of sentences under a causal LM."""

    def __init__(self, spec, tokenizer, device, bos=None, overrides=None, quant=""):
        from tokenizers import Tokenizer
        self.tok = Tokenizer.from_file(tokenizer)
        self.bos = bos if bos is not None else (self.tok.token_to_id("<|endoftext|>") or 0)
        self.device = device
        if spec.startswith("hf:"):
            from transformers import AutoModelForCausalLM

            from trenowanie_generatora_obrazkow_b200.models.frozen_lm import (refresh_rope_buffers,
                                                                              transformers5_compat)
            transformers5_compat()
            m = AutoModelForCausalLM.from_pretrained(spec[3:], dtype=torch.bfloat16, local_files_only=True,
                                                     trust_remote_code=True, **(overrides or {}))
            refresh_rope_buffers(m)
            if quant:
                from trenowanie_generatora_obrazkow_b200.models.moe_infer import patch_moe_blocks
                if not patch_moe_blocks(m, quant=quant):
                    raise ValueError(f"--quant {quant}: {spec} has no mixture-of-experts blocks")
            self.model, self.kind = m.to(device).eval(), "hf"
        else:
            if overrides or quant:
                raise ValueError("--set / --quant apply to transformers (hf:) models only")
            from trenowanie_generatora_obrazkow_b200.models.slayer import load_gpt
            self.model, self.kind = load_gpt(spec)[0].to(device).eval(), "slayer"

    def logits(self, ids):
        if self.kind == "hf":
            return self.model(input_ids=ids).logits
        return self.model(ids)

    @torch.no_grad()
    def __call__(self, sentences, batch=64):
        scores = []
        for i in range(0, len(sentences), batch):
            enc = self.tok.encode_batch(sentences[i:i + batch], add_special_tokens=False)
            seqs = [[self.bos] + e.ids for e in enc]
            L = max(len(s) for s in seqs)
            ids = torch.zeros(len(seqs), L, dtype=torch.long)
            mask = torch.zeros(len(seqs), L, dtype=torch.bool)
            for j, s in enumerate(seqs):
                ids[j, :len(s)] = torch.tensor(s)
                mask[j, 1:len(s)] = True  # every real token after BOS is predicted from its prefix
            ids, mask = ids.to(self.device), mask.to(self.device)
            logp = F.log_softmax(self.logits(ids).float(), -1)
            tok_lp = logp[:, :-1].gather(-1, ids[:, 1:, None]).squeeze(-1)
            scores += (tok_lp * mask[:, 1:]).sum(1).tolist()
        return scores


def _accuracy(groups):
    return {k: ok / n for k, (ok, n) in groups.items()}


def evaluate(scorer, pairs, batch=64, phenomena=None):
    """(overall accuracy, per-paradigm accuracy[, per-phenomenon accuracy when ``phenomena`` maps paradigms])."""
    good = scorer([g for _, g, _ in pairs], batch)
    bad = scorer([b for _, _, b in pairs], batch)
    per, by_term = {}, {}
    for (par, _, _), sg, sb in zip(pairs, good, bad):
        ok, n = per.get(par, (0, 0))
        per[par] = (ok + (sg > sb), n + 1)
        if phenomena and par in phenomena:
            ok, n = by_term.get(phenomena[par], (0, 0))
            by_term[phenomena[par]] = (ok + (sg > sb), n + 1)
    total = sum(ok for ok, _ in per.values()) / max(1, sum(n for _, n in per.values()))
    if phenomena is None:
        return total, _accuracy(per)
    return total, _accuracy(per), _accuracy(by_term)


def parse_overrides(items):
    """["k=v", ...] -> {k: JSON value of v (the raw string when it is not JSON)}."""
    out = {}
    for item in items:
        k, sep, v = item.partition("=")
        if not sep or not k:
            raise ValueError(f"--set wants KEY=VALUE, got {item!r}")
        try:
            out[k] = json.loads(v)
        except json.JSONDecodeError:
            out[k] = v
    return out


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("models", nargs="+")
    p.add_argument("--data", required=True)
    p.add_argument("--tokenizer", required=True, help="tokenizer.json of the models")
    p.add_argument("--limit", type=int, default=0)
    p.add_argument("--batch", type=int, default=64)
    p.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    p.add_argument("--out", default=None)
    p.add_argument("--quant", choices=["", "int8"], default="",
                   help="transformers MoE models: int8 expert weights through the fused expert path")
    p.add_argument("--set", nargs="*", default=[], metavar="KEY=VALUE",
                   help="config overrides for transformers models, e.g. num_experts_per_tok=16")
    a = p.parse_args(argv)
    overrides = parse_overrides(a.set)
    phenomena = {}
    pairs = load_pairs(a.data, a.limit, phenomena)
    print(f"{len(pairs)} pairs, {len({q for q, _, _ in pairs})} paradigms")
    results = {}
    for spec in a.models:
        t0 = time.time()
        total, per, terms = evaluate(Scorer(spec, a.tokenizer, a.device, overrides=overrides, quant=a.quant), pairs,
                                     a.batch, phenomena)
        key = spec + (f" {overrides}" if overrides else "") + (f" {a.quant}" if a.quant else "")
        results[key] = dict(accuracy=total, paradigms=per, **({"phenomena": terms} if terms else {}))
        print(f"{key}: {100 * total:.1f} % ({time.time() - t0:.0f} s)")
        for k, v in sorted(terms.items()):
            print(f"  {k:28s} {100 * v:5.1f}")
    if a.out:
        with open(a.out, "w") as f:
            json.dump(results, f, indent=1)
    return results


if __name__ == "__main__":
    main()
