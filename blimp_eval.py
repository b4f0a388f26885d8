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
"""
import argparse
import glob
import json
import os
import time

import torch
import torch.nn.functional as F


def load_pairs(data, limit=0):
    """[(paradigm, good, bad)] from the files under ``data``."""
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
    return out


class Scorer:
    """Summed token log-probabilities of sentences under a causal LM."""

    def __init__(self, spec, tokenizer, device, bos=None):
        from tokenizers import Tokenizer
        self.tok = Tokenizer.from_file(tokenizer)
        self.bos = bos if bos is not None else (self.tok.token_to_id("<|endoftext|>") or 0)
        self.device = device
        if spec.startswith("hf:"):
            from transformers import AutoModelForCausalLM
            m = AutoModelForCausalLM.from_pretrained(spec[3:], torch_dtype=torch.bfloat16, local_files_only=True,
                                                     trust_remote_code=True)
            self.model, self.kind = m.to(device).eval(), "hf"
        else:
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


def evaluate(scorer, pairs, batch=64):
    good = scorer([g for _, g, _ in pairs], batch)
    bad = scorer([b for _, _, b in pairs], batch)
    per = {}
    for (par, _, _), sg, sb in zip(pairs, good, bad):
        ok, n = per.get(par, (0, 0))
        per[par] = (ok + (sg > sb), n + 1)
    acc = {k: ok / n for k, (ok, n) in per.items()}
    total = sum(ok for ok, _ in per.values()) / max(1, sum(n for _, n in per.values()))
    return total, acc


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("models", nargs="+")
    p.add_argument("--data", required=True)
    p.add_argument("--tokenizer", required=True, help="tokenizer.json of the models")
    p.add_argument("--limit", type=int, default=0)
    p.add_argument("--batch", type=int, default=64)
    p.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    p.add_argument("--out", default=None)
    a = p.parse_args(argv)
    pairs = load_pairs(a.data, a.limit)
    print(f"{len(pairs)} pairs, {len({q for q, _, _ in pairs})} paradigms")
    results = {}
    for spec in a.models:
        t0 = time.time()
        total, per = evaluate(Scorer(spec, a.tokenizer, a.device), pairs, a.batch)
        results[spec] = dict(accuracy=total, paradigms=per)
        print(f"{spec}: {100 * total:.1f} % ({time.time() - t0:.0f} s)")
    if a.out:
        with open(a.out, "w") as f:
            json.dump(results, f, indent=1)
    return results


if __name__ == "__main__":
    main()
