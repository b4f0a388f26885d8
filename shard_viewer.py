"""Browse prepared training shards in a web browser (the role of the reference's tests/shard_viewer.py, for this
project's shard layout; standard library + numpy + PIL, no network).

  python shard_viewer.py --root data/aurora [--img-root data/flux_reason_1024] --port 8765
  # then open http://localhost:8765 (on a remote box: ssh -L 8765:localhost:8765 ...)

Pages: the shard list (images, caption rows, which latent / token / caption / image files exist), a paged grid per
shard (thumbnails with their captions, filtered by a caption substring), and one image with every caption (English
and translated) and its latent shapes. Images are the packed originals (<shard>.img.bin) when there are any, else a
false-colour preview of the 256 px latents (three channel groups; not a decoded image).
"""
import argparse
import html
import io
import json
import os
import urllib.parse
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer

import numpy as np

PER_PAGE = 60
STYLE = ("body{font:14px system-ui,sans-serif;margin:0;background:#fafaf8;color:#222}"
         "header{padding:8px 14px;border-bottom:1px solid #ddd;background:#fff;position:sticky;top:0}"
         "main{padding:14px}table{border-collapse:collapse}td,th{padding:3px 10px;border-bottom:1px solid #eee}"
         ".grid{display:grid;grid-template-columns:repeat(auto-fill,minmax(220px,1fr));gap:12px}"
         ".cell{background:#fff;border:1px solid #e4e4e0;border-radius:6px;padding:6px}"
         ".cell img{width:100%;image-rendering:pixelated}.cap{font-size:12px;color:#444;margin-top:4px}"
         "a{color:#2457c5;text-decoration:none}")
MAGIC = ((b"\xff\xd8\xff", "image/jpeg"), (b"\x89PNG", "image/png"), (b"RIFF", "image/webp"), (b"GIF8", "image/gif"))


class ShardSet:
    """Read-only view of a data directory (and an optional packed-image directory)."""

    def __init__(self, root, img_root=""):
        self.root, self.img_root = root, img_root or root
        files = set(os.listdir(root))
        self.names = sorted(f[: -len(".off.npy")] for f in files if f.endswith(".off.npy")
                            and not f.endswith(".img.off.npy"))
        if not self.names:  # image-only directory
            self.names = sorted(f[: -len(".img.off.npy")] for f in os.listdir(self.img_root)
                                if f.endswith(".img.off.npy"))

    def _p(self, name, suffix, root=None):
        return os.path.join(root or self.root, f"{name}.{suffix}")

    def kinds(self, name):
        pre = name + "."
        out = sorted(f[len(pre):] for f in os.listdir(self.root) if f.startswith(pre))
        if self.img_root != self.root:
            out += sorted(f[len(pre):] for f in os.listdir(self.img_root) if f.startswith(pre) and ".img." in f)
        return out

    def has_images(self, name):
        return os.path.exists(self._p(name, "img.off.npy", self.img_root))

    def count(self, name):
        if self.has_images(name):
            return len(np.load(self._p(name, "img.off.npy", self.img_root), mmap_mode="r")) - 1
        if os.path.exists(self._p(name, "off.npy")):
            return len(np.load(self._p(name, "off.npy"), mmap_mode="r")) - 1
        return 0

    def captions(self, name):
        """{lang: [[captions of image i]]} from <name>.caps.json and <name>.caps_<lang>.json."""
        out = {}
        for f in sorted(os.listdir(self.root)):
            if f.startswith(name + ".caps") and f.endswith(".json") and not f.endswith(".stats.json"):
                lang = f[len(name) + len(".caps"):-len(".json")].lstrip("_") or "en"
                with open(os.path.join(self.root, f), encoding="utf-8") as fh:
                    out[lang] = json.load(fh)
        return out

    def image(self, name, i):
        """(bytes, content type) of image i: the packed original, or a PNG latent preview."""
        if self.has_images(name):
            off = np.load(self._p(name, "img.off.npy", self.img_root), mmap_mode="r")
            with open(self._p(name, "img.bin", self.img_root), "rb") as f:
                f.seek(int(off[i]))
                data = f.read(int(off[i + 1] - off[i]))
            return data, next((t for m, t in MAGIC if data.startswith(m)), "application/octet-stream")
        import torch
        from PIL import Image

        from sample_ckpt import latent_preview
        lat = np.load(self._p(name, "lat.npy"), mmap_mode="r")
        img = latent_preview(torch.from_numpy(np.array(lat[i:i + 1], dtype=np.float32)))[0]
        buf = io.BytesIO()
        Image.fromarray(img).resize((img.shape[1] * 8, img.shape[0] * 8), Image.NEAREST).save(buf, format="PNG")
        return buf.getvalue(), "image/png"

    def latent_shapes(self, name):
        out = {}
        for k in self.kinds(name):
            if k.startswith("lat") and k.endswith(".npy"):
                out[k[:-4]] = list(np.load(self._p(name, k), mmap_mode="r").shape[1:])
        return out


def _page(title, body):
    return (f"<!doctype html><html><head><meta charset='utf-8'><title>{html.escape(title)}</title>"
            f"<style>{STYLE}</style></head><body><header><a href='/'>shards</a> &middot; {html.escape(title)}"
            f"</header><main>{body}</main></body></html>")


def render_index(ss):
    rows = "".join(f"<tr><td><a href='/shard?name={urllib.parse.quote(n)}'>{html.escape(n)}</a></td>"
                   f"<td>{ss.count(n)}</td><td>{html.escape(' '.join(ss.kinds(n)))}</td></tr>" for n in ss.names)
    return _page(f"{len(ss.names)} shards in {ss.root}",
                 f"<table><tr><th>shard</th><th>images</th><th>files</th></tr>{rows}</table>")


def render_shard(ss, name, page=0, q=""):
    caps = ss.captions(name)
    n = ss.count(name)
    first = caps.get("en") or next(iter(caps.values()), [])
    idx = [i for i in range(n) if not q or any(q.lower() in c.lower() for lang in caps.values()
                                                if i < len(lang) for c in lang[i])]
    pages = max(1, -(-len(idx) // PER_PAGE))
    page = min(max(0, page), pages - 1)
    cells = []
    for i in idx[page * PER_PAGE:(page + 1) * PER_PAGE]:
        cap = first[i][0] if i < len(first) and first[i] else ""
        link = f"/item?name={urllib.parse.quote(name)}&i={i}"
        cells.append(f"<div class='cell'><a href='{link}'><img loading='lazy' src='/img?name="
                     f"{urllib.parse.quote(name)}&i={i}'></a><div class='cap'>#{i} {html.escape(cap[:240])}</div></div>")
    qs = urllib.parse.quote(q)
    nav = " ".join(f"<a href='/shard?name={urllib.parse.quote(name)}&page={p}&q={qs}'>{'[' if p == page else ''}"
                   f"{p + 1}{']' if p == page else ''}</a>" for p in range(pages))
    form = (f"<form action='/shard'><input type='hidden' name='name' value='{html.escape(name)}'>"
            f"<input name='q' value='{html.escape(q)}' placeholder='caption contains'> <button>filter</button></form>")
    return _page(f"{name}: {len(idx)} of {n} images", f"{form}<p>{nav}</p><div class='grid'>{''.join(cells)}</div>")


def render_item(ss, name, i):
    caps = ss.captions(name)
    lists = "".join(f"<h4>{html.escape(lang)}</h4><ol>" + "".join(f"<li>{html.escape(c)}</li>" for c in rows[i])
                    + "</ol>" for lang, rows in caps.items() if i < len(rows))
    shapes = html.escape(json.dumps(ss.latent_shapes(name)))
    return _page(f"{name} #{i}", f"<img style='max-width:90vw;image-rendering:pixelated' src='/img?name="
                                 f"{urllib.parse.quote(name)}&i={i}'><p>latents: {shapes}</p>{lists}")


def make_handler(ss):
    class Handler(BaseHTTPRequestHandler):
        def log_message(self, *a):
            pass

        def _send(self, body, ctype="text/html; charset=utf-8", code=200):
            data = body.encode() if isinstance(body, str) else body
            self.send_response(code)
            self.send_header("Content-Type", ctype)
            self.send_header("Content-Length", str(len(data)))
            self.end_headers()
            self.wfile.write(data)

        def do_GET(self):
            url = urllib.parse.urlparse(self.path)
            qs = {k: v[0] for k, v in urllib.parse.parse_qs(url.query).items()}
            name = qs.get("name", "")
            try:
                if url.path == "/":
                    return self._send(render_index(ss))
                if name not in ss.names:
                    return self._send(_page("not found", "no such shard"), code=404)
                if url.path == "/shard":
                    return self._send(render_shard(ss, name, int(qs.get("page", 0)), qs.get("q", "")))
                i = int(qs.get("i", -1))
                if not 0 <= i < ss.count(name):
                    return self._send(_page("not found", "no such image"), code=404)
                if url.path == "/img":
                    data, ctype = ss.image(name, i)
                    return self._send(data, ctype)
                if url.path == "/item":
                    return self._send(render_item(ss, name, i))
                return self._send(_page("not found", "unknown page"), code=404)
            except (OSError, ValueError) as e:
                return self._send(_page("error", html.escape(str(e))), code=500)
    return Handler


def serve(root, img_root="", host="127.0.0.1", port=8765):
    """A ThreadingHTTPServer over the shards (port 0 picks a free one: server.server_address)."""
    return ThreadingHTTPServer((host, port), make_handler(ShardSet(root, img_root)))


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--root", required=True, help="shard directory (latents, token rows, captions)")
    p.add_argument("--img-root", default="", help="packed images (<shard>.img.bin) when kept elsewhere")
    p.add_argument("--host", default="127.0.0.1")
    p.add_argument("--port", type=int, default=8765)
    a = p.parse_args(argv)
    server = serve(a.root, a.img_root, a.host, a.port)
    print(f"serving {a.root} on http://{a.host}:{server.server_address[1]}", flush=True)
    try:
        server.serve_forever()
    except KeyboardInterrupt:
        pass
    finally:
        server.server_close()


if __name__ == "__main__":
    main()
