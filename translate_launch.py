"""Run caption translation on several GPUs with automatic restarts (the role of the reference's translate_tmux.sh,
without tmux): one translate_captions.py worker per GPU (CUDA_VISIBLE_DEVICES=<gpu>, --rank i --world N), each
restarted after a crash, and a progress line of finished shards every --progress-every seconds. Finished shards are
skipped by the workers, so running the launcher again after a crash or a reboot continues where it stopped (only the
shards in progress are redone).

  python translate_launch.py --gpus 0 1 2 3 4 5 6 7 --data data/aurora_full
  python translate_launch.py --gpus 0 1 --parquet-dir data/monet_z_image --python .venv-vllm/bin/python \\
      --log-dir logs/translate -- --max-tokens 768 --gpu-mem 0.9
  # at boot (crontab -e):  @reboot cd /path/to/repo && python translate_launch.py --gpus 0 1 2 3 --data data/x

Arguments after `--` go to every worker. Worker output goes to <log-dir>/gpu<i>.log (appended across restarts) or,
without --log-dir, to this terminal. --max-restarts bounds the restarts per worker (0 = no bound). On Ctrl-C or
SIGTERM the launcher stops the workers it started (each worker's own process group) and exits.
"""
import argparse
import glob
import os
import signal
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))


def progress(data="", parquet_dir="", suffix="pl"):
    """(finished, total) shards: <shard>.caps_<suffix>.json per <shard>.caps.json, or <file>.<suffix>.parquet per
    source parquet."""
    if data:
        total = len(glob.glob(os.path.join(data, "*.caps.json")))
        done = len(glob.glob(os.path.join(data, f"*.caps_{suffix}.json")))
        return done, total
    ext = f".{suffix}.parquet"
    files = glob.glob(os.path.join(parquet_dir, "**", "*.parquet"), recursive=True)
    done = sum(f.endswith(ext) for f in files)
    return done, len(files) - done


class Worker:
    def __init__(self, index, gpu, cmd, log_path=None):
        self.index, self.gpu, self.cmd, self.log_path = index, gpu, cmd, log_path
        self.proc, self.restarts, self.done, self.next_start = None, 0, False, 0.0

    def start(self):
        env = dict(os.environ, CUDA_VISIBLE_DEVICES=str(self.gpu))
        out = open(self.log_path, "a") if self.log_path else None
        self.proc = subprocess.Popen(self.cmd, cwd=ROOT, env=env, stdout=out,
                                     stderr=subprocess.STDOUT if out else None, start_new_session=True)
        if out:
            out.close()

    def stop(self):
        if self.proc is not None and self.proc.poll() is None:
            try:
                os.killpg(self.proc.pid, signal.SIGTERM)  # the worker's own process group (its engine's children)
            except ProcessLookupError:
                pass
            try:
                self.proc.wait(timeout=30)
            except subprocess.TimeoutExpired:
                os.killpg(self.proc.pid, signal.SIGKILL)
                self.proc.wait()


def worker_command(python, script, rank, world, data, parquet_dir, extra):
    src = ["--data", data] if data else ["--parquet-dir", parquet_dir]
    return [python, script, *src, "--rank", str(rank), "--world", str(world), *extra]


def run(workers, restart_delay=30.0, max_restarts=0, poll=1.0, progress_every=60.0, report=None, log=print):
    """Supervise until every worker exits 0 (or runs out of restarts). Returns {index: last exit code}."""
    for w in workers:
        w.start()
    codes, last_report = {}, time.time()
    while True:
        now = time.time()
        for w in workers:
            if w.done:
                continue
            if w.proc is None:
                if now >= w.next_start:
                    w.start()
                continue
            rc = w.proc.poll()
            if rc is None:
                continue
            codes[w.index] = rc
            w.proc = None
            if rc == 0:
                w.done = True
                log(f"worker {w.index} (GPU {w.gpu}) finished")
            elif max_restarts and w.restarts >= max_restarts:
                w.done = True
                log(f"worker {w.index} (GPU {w.gpu}) exited with {rc}; no restarts left")
            else:
                w.restarts += 1
                w.next_start = now + restart_delay
                log(f"worker {w.index} (GPU {w.gpu}) exited with {rc}; restart {w.restarts} in {restart_delay:g} s")
        if all(w.done for w in workers):
            return codes
        if report is not None and now - last_report >= progress_every:
            done, total = report()
            log(f"{done} / {total} shards translated ({time.strftime('%H:%M:%S')})")
            last_report = now
        time.sleep(poll)


def main(argv=None):
    argv = list(sys.argv[1:] if argv is None else argv)
    extra = []
    if "--" in argv:
        i = argv.index("--")
        argv, extra = argv[:i], argv[i + 1:]
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", nargs="+", required=True, help="GPU indices, one worker each")
    p.add_argument("--data", default="")
    p.add_argument("--parquet-dir", default="")
    p.add_argument("--suffix", default="pl")
    p.add_argument("--python", default=sys.executable, help="interpreter of the workers (e.g. a vLLM environment)")
    p.add_argument("--script", default=os.path.join(ROOT, "translate_captions.py"))
    p.add_argument("--log-dir", default="")
    p.add_argument("--restart-delay", type=float, default=30.0)
    p.add_argument("--max-restarts", type=int, default=0)
    p.add_argument("--progress-every", type=float, default=60.0)
    a = p.parse_args(argv)
    if bool(a.data) == bool(a.parquet_dir):
        p.error("give --data or --parquet-dir")
    if a.log_dir:
        os.makedirs(a.log_dir, exist_ok=True)
    world = len(a.gpus)
    workers = [Worker(i, g, worker_command(a.python, a.script, i, world, a.data, a.parquet_dir, extra),
                      os.path.join(a.log_dir, f"gpu{g}.log") if a.log_dir else None) for i, g in enumerate(a.gpus)]

    def stop(signum, frame):
        for w in workers:
            w.stop()
        sys.exit(128 + signum)

    previous = signal.signal(signal.SIGTERM, stop)
    try:
        codes = run(workers, a.restart_delay, a.max_restarts, progress_every=a.progress_every,
                    report=lambda: progress(a.data, a.parquet_dir, a.suffix), log=lambda s: print(s, flush=True))
    except KeyboardInterrupt:
        for w in workers:
            w.stop()
        raise
    finally:
        signal.signal(signal.SIGTERM, previous)
    done, total = progress(a.data, a.parquet_dir, a.suffix)
    print(f"{done} / {total} shards translated; exit codes {codes}", flush=True)
    return codes


if __name__ == "__main__":
    main()
