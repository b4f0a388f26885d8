"""Run logging: stdout lines plus optional wandb (reference train.py:509-537).

wandb is used only when it is importable and has credentials (API key, offline mode or a netrc entry); the run id
is persisted in <out>/wandb_id.txt so a resumed run continues the same wandb run. A JSON-lines copy of every logged
dict goes to <out>/log.jsonl either way.
"""
import json
import os
import uuid


def wandb_available():
    try:
        import wandb  # noqa: F401
    except ImportError:
        return False
    if os.environ.get("WANDB_API_KEY") or os.environ.get("WANDB_MODE") in ("offline", "dryrun"):
        return True
    import netrc
    from urllib.parse import urlparse
    host = urlparse(os.environ.get("WANDB_BASE_URL", "https://api.wandb.ai")).hostname
    try:
        return netrc.netrc(os.environ.get("NETRC")).authenticators(host) is not None
    except (FileNotFoundError, netrc.NetrcParseError):
        return False


class RunLogger:
    def __init__(self, out_dir, config, enabled=True, project="trenowanie_generatora_obrazkow"):
        self.out_dir = out_dir
        self.enabled = enabled
        self.wb = None
        if enabled:
            os.makedirs(out_dir, exist_ok=True)
        self.jsonl = open(os.path.join(out_dir, "log.jsonl"), "a") if enabled else None
        if enabled and wandb_available():
            import wandb
            id_path = os.path.join(out_dir, "wandb_id.txt")
            run_id = open(id_path).read().strip() if os.path.exists(id_path) else uuid.uuid4().hex[:12]
            with open(id_path, "w") as f:
                f.write(run_id)
            self.wb = wandb.init(project=project, id=run_id, resume="allow", dir=out_dir,
                                 name=os.path.basename(os.path.normpath(out_dir)))
            self.wb.config.update({k: v for k, v in config.items() if isinstance(v, (int, float, str, bool))},
                                  allow_val_change=True)

    def log(self, stats, step):
        if not self.enabled:
            return
        self.jsonl.write(json.dumps(dict(stats, step=step)) + "\n")
        self.jsonl.flush()
        if self.wb is not None:
            self.wb.log(stats, step=step)

    def close(self):
        if self.jsonl is not None:
            self.jsonl.close()
        if self.wb is not None:
            self.wb.finish()
