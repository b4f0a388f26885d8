"""Caption translation for the Polish text encoders (reference translate_captions.py, translate_tmux.sh): a local
machine-translation model served by vLLM's offline engine turns

  --data DIR         <shard>.caps.json (per image a list of captions) -> <shard>.caps_<suffix>.json, same structure
                     and order, so the shard's latents and offsets stay valid and prepare_data.py tokenizes it
  --parquet-dir DIR  prepare_monet.py parquets (one caption per row in --column) -> <file>.<suffix>.parquet next to
                     each, with `__key__` and `<column>_<suffix>` in the same row order (empty captions stay empty)

  python translate_captions.py --data data/aurora --model models/Index-Translate-2B --pilot 2000
  for i in 0 1 2 3 4 5 6 7; do CUDA_VISIBLE_DEVICES=$i python translate_captions.py --data data/aurora \\
      --model models/Index-Translate-2B --rank $i --world 8 > translate_$i.log 2>&1 & done

Text in double quotes is what is written in the image ("a sign that says 'OPEN'"): those spans are swapped for
numbered placeholders before translation and put back afterwards, so the caption keeps matching the image; a caption
whose placeholders do not come back exactly once each is translated again without them. Unique captions are
translated once per shard; a caption whose prompt does not fit the context is left untranslated (None). Outputs that
look wrong (CJK characters, a length far from the source's) are counted as flagged. Every shard is written to a
temporary name and renamed, with per-shard counters in a .stats.json; a rerun skips finished shards (the restart
loop of the reference's tmux script is this skip). The model weights must be local (no network here).
"""
import argparse
import glob
import json
import os
import random
import re
import time

PROMPT = "Translate the following {src} text into {tgt}. Output only the translation.\n\n{text}"
QUOTED = re.compile(r'"[^"\n]{1,80}"|“[^”\n]{1,80}”|„[^”"\n]{1,80}[”"]')
HOLDER = "<<{}>>"
CJK = re.compile(r"[぀-ヿ㐀-鿿]")
LEAD_EN = re.compile(r"^(?:(?:the|this) (?:image|picture|photo(?:graph)?|illustration) (?:shows|depicts|features|"
                     r"captures|presents|displays|showcases|is(?: of)?)|in (?:this|the) (?:image|picture),? "
                     r"(?:we (?:can )?see|there (?:is|are)))\s+", re.I)


def strip_lead(text):
    """Drop a leading 'The image shows' style phrase (captioner boilerplate) and capitalise what follows."""
    if not text:
        return text
    out = LEAD_EN.sub("", text.strip(), count=1)
    return out[:1].upper() + out[1:] if out else text


def protect(text):
    """Quoted spans -> <<0>>, <<1>>, ...; returns (text, spans)."""
    spans = []

    def repl(m):
        spans.append(m.group(0))
        return HOLDER.format(len(spans) - 1)
    return QUOTED.sub(repl, text), spans


def restore(text, spans):
    """Spans back in place of their placeholders; None unless every placeholder occurs exactly once."""
    for i, span in enumerate(spans):
        if text.count(HOLDER.format(i)) != 1:
            return None
        text = text.replace(HOLDER.format(i), span)
    return None if re.search(r"<<\d+>>", text) else text


def looks_wrong(src, out):
    return not out or CJK.search(out) is not None or not 0.4 <= len(out) / max(1, len(src)) <= 3.0


class Translator:
    """generate(prompts) -> texts (the engine); count(text) -> tokens (the context check)."""

    def __init__(self, generate, make_prompt, count=None, max_in=3328):
        self.generate, self.make_prompt, self.count, self.max_in = generate, make_prompt, count, max_in

    def __call__(self, texts):
        prot = [protect(t) for t in texts]
        prompts = [self.make_prompt(pt) for pt, _ in prot]
        fits = [self.count is None or self.count(p) <= self.max_in for p in prompts]
        idx = [i for i, f in enumerate(fits) if f]
        outs = [None] * len(texts)
        for i, o in zip(idx, self.generate([prompts[i] for i in idx])):
            outs[i] = o.strip()
        res, retry = [], []
        st = dict(captions=len(texts), quoted=sum(bool(s) for _, s in prot), retried=0, flagged=0,
                  too_long=len(texts) - len(idx))
        for i, ((_, spans), out) in enumerate(zip(prot, outs)):
            r = out if out is None or not spans else restore(out, spans)
            if out is not None and r is None:
                retry.append(i)
            res.append(r)
        if retry:  # placeholders lost or duplicated: translate the original text
            st["retried"] = len(retry)
            for i, out in zip(retry, self.generate([self.make_prompt(texts[i]) for i in retry])):
                res[i] = out.strip()
        st["flagged"] = sum(r is not None and looks_wrong(t, r) for t, r in zip(texts, res))
        return res, st


def _atomic_json(path, obj):
    with open(path + ".tmp", "w") as f:
        json.dump(obj, f, ensure_ascii=False)
    os.replace(path + ".tmp", path)


def translate_caps(data, translate, suffix="pl", rank=0, world=1, log=print):
    shards = sorted(glob.glob(os.path.join(data, "*.caps.json")))[rank::world]
    for n, path in enumerate(shards):
        out = path.replace(".caps.json", f".caps_{suffix}.json")
        if os.path.exists(out):
            continue
        t0 = time.time()
        caps = json.load(open(path))
        uniq = list(dict.fromkeys(c for img in caps for c in img))
        res, st = translate(uniq)
        table = dict(zip(uniq, res))
        _atomic_json(out, [[table[c] for c in img] for img in caps])
        _atomic_json(out.replace(".json", ".stats.json"), st)
        log(f"[{n + 1}/{len(shards)}] {os.path.basename(path)}: {st} {len(uniq) / max(time.time() - t0, 1e-9):.1f} "
            "captions/s")


def translate_parquets(root, translate, column="caption_short", suffix="pl", rank=0, world=1, strip=False,
                       log=print):
    import pyarrow as pa
    import pyarrow.parquet as pq
    ext = f".{suffix}.parquet"
    files = sorted(f for f in glob.glob(os.path.join(root, "**", "*.parquet"), recursive=True)
                   if not f.endswith(ext))[rank::world]
    for n, path in enumerate(files):
        out = path[: -len(".parquet")] + ext
        if os.path.exists(out):
            continue
        src = pq.read_table(path, columns=["__key__", column])
        texts = [strip_lead(c) if strip else c for c in src[column].to_pylist()]
        uniq = list(dict.fromkeys(c for c in texts if c))
        res, st = translate(uniq)
        table = dict(zip(uniq, res))
        pq.write_table(pa.table({"__key__": src["__key__"],
                                 f"{column}_{suffix}": pa.array([table.get(c) if c else None for c in texts],
                                                                pa.string())}), out + ".tmp", compression="zstd")
        os.replace(out + ".tmp", out)
        _atomic_json(out[: -len(".parquet")] + ".stats.json", st)
        log(f"[{n + 1}/{len(files)}] {os.path.relpath(path, root)}: {st}")


def vllm_translator(model, src, tgt, max_tokens=768, gpu_mem=0.85, max_num_seqs=1024, max_batched=16384):
    from transformers import AutoTokenizer
    from vllm import LLM, SamplingParams
    tok = AutoTokenizer.from_pretrained(model, local_files_only=True)
    llm = LLM(model, gpu_memory_utilization=gpu_mem, max_model_len=4096, enable_prefix_caching=True,
              max_num_seqs=max_num_seqs, max_num_batched_tokens=max_batched)
    params = SamplingParams(temperature=0.0, max_tokens=max_tokens)

    def make_prompt(text):
        msg = [{"role": "user", "content": PROMPT.format(src=src, tgt=tgt, text=text)}]
        return tok.apply_chat_template(msg, tokenize=False, add_generation_prompt=True)

    def generate(prompts):
        return [o.outputs[0].text for o in llm.generate(prompts, params)] if prompts else []

    return Translator(generate, make_prompt, lambda p: len(tok(p, add_special_tokens=False).input_ids),
                      4096 - max_tokens)


def main(argv=None, translator=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--data", default="")
    p.add_argument("--parquet-dir", default="")
    p.add_argument("--column", default="caption_short")
    p.add_argument("--strip-prefix", action="store_true", help="--parquet-dir: drop 'The image shows' first")
    p.add_argument("--model", default="models/Index-Translate-2B", help="local model directory")
    p.add_argument("--src", default="English")
    p.add_argument("--tgt", default="Polish")
    p.add_argument("--suffix", default="pl")
    p.add_argument("--rank", type=int, default=0)
    p.add_argument("--world", type=int, default=1)
    p.add_argument("--max-tokens", type=int, default=768)
    p.add_argument("--pilot", type=int, default=0, help="translate this many captions of the first shard, print pairs")
    p.add_argument("--gpu-mem", type=float, default=0.85, help="fraction of GPU memory the engine may take")
    p.add_argument("--max-num-seqs", type=int, default=1024, help="sequences decoded at once (engine default 256)")
    p.add_argument("--max-batched-tokens", type=int, default=16384, help="tokens per scheduler step (prefill chunk)")
    a = p.parse_args(argv)
    assert bool(a.data) != bool(a.parquet_dir), "give --data or --parquet-dir"
    translate = translator or vllm_translator(a.model, a.src, a.tgt, a.max_tokens, a.gpu_mem, a.max_num_seqs,
                                              a.max_batched_tokens)
    if a.pilot:
        if a.data:
            caps = json.load(open(sorted(glob.glob(os.path.join(a.data, "*.caps.json")))[0]))
            flat = list(dict.fromkeys(c for img in caps for c in img))[: a.pilot]
        else:
            import pyarrow.parquet as pq
            f = sorted(glob.glob(os.path.join(a.parquet_dir, "**", "*.parquet"), recursive=True))[0]
            flat = [c for c in pq.read_table(f, columns=[a.column])[a.column].to_pylist() if c][: a.pilot]
        t0 = time.time()
        res, st = translate(flat)
        print(json.dumps(st), f"{len(flat) / max(time.time() - t0, 1e-9):.1f} captions/s")
        random.seed(0)
        for i in random.sample(range(len(flat)), min(15, len(flat))):
            print(f"\n{a.src}: {flat[i]}\n{a.tgt}: {res[i]}")
        return
    if a.data:
        translate_caps(a.data, translate, a.suffix, a.rank, a.world)
    else:
        translate_parquets(a.parquet_dir, translate, a.column, a.suffix, a.rank, a.world, a.strip_prefix)


if __name__ == "__main__":
    main()
