"""Small web UI for an exported model, reachable from a phone on the same network (reference app.py, which uses
Gradio; Gradio is not installed here, so this is a FastAPI page with the same controls: prompt, steps, guidance,
seed, resolution).

  python app.py --model exports/homeimg                    # a local export directory (utils/export.py layout)
  python app.py --model exports/homeimg --port 7860

Open http://<this machine's LAN IP>:7860 (printed at startup). GET / serves the form; POST /generate with JSON
{"prompt", "steps", "guidance", "seed", "res", "count"} returns a PNG: the decoded image when the export carries a FLUX.2 VAE
(and diffusers is importable), otherwise a false-colour preview of the latents.
"""
import argparse
import io
import random
import socket

EXAMPLES = [
    "a red fox sitting in a snowy forest at sunrise, photograph",
    "a watercolor painting of a lighthouse on a rocky coast",
    "a small robot reading a book in a cozy library",
    "rudy lis siedzący w zaśnieżonym lesie o wschodzie słońca, fotografia",
]

PAGE = """<!doctype html><html><head><meta name="viewport" content="width=device-width, initial-scale=1">
<title>HomeIMG</title></head><body style="font-family:sans-serif;max-width:640px;margin:auto">
<h3>HomeIMG</h3>
<textarea id="p" rows="3" style="width:100%">{example}</textarea><br>
steps <input id="s" type="number" value="{steps}" min="1" max="100">
guidance <input id="g" type="number" value="{guidance}" step="0.5">
seed <input id="d" type="number" value="-1">
res <select id="r">{res_options}</select>
images <input id="n" type="number" value="1" min="1" max="8">
<button onclick="go()">generate</button><br><img id="o" style="width:100%;margin-top:8px">
<script>
async function go() {{
  const body = {{prompt: p.value, steps: +s.value, guidance: +g.value, seed: +d.value, res: +r.value,
                 count: +document.getElementById('n').value}};
  const resp = await fetch('/generate', {{method: 'POST', headers: {{'Content-Type': 'application/json'}},
                                         body: JSON.stringify(body)}});
  o.src = URL.createObjectURL(await resp.blob());
}}
</script></body></html>"""


def lan_ip():
    try:
        with socket.socket(socket.AF_INET, socket.SOCK_DGRAM) as s:
            s.connect(("10.255.255.255", 1))  # no packet is sent; picks the outgoing interface
            return s.getsockname()[0]
    except OSError:
        return "127.0.0.1"


def build_app(pipe, default_res=1024, steps=30, guidance=3.0):
    import numpy as np
    import torch
    from fastapi import FastAPI
    from fastapi.responses import HTMLResponse, Response
    from PIL import Image
    from pydantic import BaseModel

    from sample_ckpt import latent_preview

    d_steps, d_guidance, d_res = steps, guidance, default_res

    class Req(BaseModel):
        prompt: str
        steps: int = d_steps
        guidance: float = d_guidance
        seed: int = -1
        res: int = d_res
        count: int = 1  # images of the prompt (1-8), one noise draw each, returned as one grid

    app = FastAPI()
    options = "".join(f'<option value="{r}"{" selected" if r == default_res else ""}>{r}</option>'
                      for r in (256, 512, 768, 1024) if r <= max(default_res, 256))

    @app.get("/", response_class=HTMLResponse)
    def index():
        return PAGE.format(example=random.choice(EXAMPLES), steps=steps, guidance=guidance, res_options=options)

    @app.post("/generate")
    def generate(req: Req):
        seed = req.seed if req.seed >= 0 else random.randrange(2 ** 31)
        n = max(1, min(int(req.count), 8))
        with torch.no_grad():
            out = pipe([req.prompt] * n, height=req.res, num_inference_steps=max(1, min(req.steps, 100)),
                       guidance_scale=req.guidance, seed=seed)
        imgs = [np.asarray(i) for i in (out.images if out.images is not None else latent_preview(out.latents))]
        cols = min(n, 4)
        h, w = imgs[0].shape[:2]
        grid = np.zeros((-(-n // cols) * h, cols * w, 3), dtype=np.uint8)
        for k, im in enumerate(imgs):  # up to 4 per row
            grid[(k // cols) * h:(k // cols + 1) * h, (k % cols) * w:(k % cols + 1) * w] = im
        buf = io.BytesIO()
        Image.fromarray(grid).save(buf, format="PNG")
        return Response(buf.getvalue(), media_type="image/png", headers={"X-Seed": str(seed)})

    return app


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--model", required=True, help="export directory")
    p.add_argument("--port", type=int, default=7860)
    p.add_argument("--host", default="0.0.0.0")
    p.add_argument("--gpu", type=int, default=0)
    p.add_argument("--res", type=int, default=1024)
    p.add_argument("--cfg", type=float, default=3.0, help="default guidance value of the page; 1 for guidance-distilled "
                   "models (train_pp.py --dance-opd / --diffusion-opd)")
    a = p.parse_args(argv)
    import torch
    import uvicorn

    from trenowanie_generatora_obrazkow_b200.sampling.pipeline import HomeIMGPipeline
    device = f"cuda:{a.gpu}" if torch.cuda.is_available() else "cpu"
    pipe = HomeIMGPipeline.from_pretrained(a.model, device=device)
    print(f"serving {a.model} on http://{lan_ip()}:{a.port}", flush=True)
    uvicorn.run(build_app(pipe, a.res, guidance=a.cfg), host=a.host, port=a.port)


if __name__ == "__main__":
    main()
