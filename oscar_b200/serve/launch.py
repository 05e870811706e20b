"""One-shot launch with gates: ``python -m oscar_b200.serve.launch --gpus 4 [serve options]``.

The stages of the reference's installer (``delivery/install_and_launch.sh:51-272``),
for this framework:

1. self-check - versions, the sm_100a extension, the GPUs (``utils/platform``); a
   mismatch stops the launch;
2. fingerprint - sha256 of the package source, expected in every rank's READY manifest;
3. rotations - reuse ``--rotations`` (default ``OSCAR_ASCEND_K_ROTATION_PATH`` or
   ``oscar_rotations.pt``) when it is a v2 checkpoint, else calibrate one with
   ``oscar_b200.kv.gen_rotations`` on the same GPUs (``--no-calibrate``: seeded random
   rotations); the serve processes get it through ``OSCAR_ASCEND_K/V_ROTATION_PATH``;
4. probes - ``oscar_b200.serve.probes`` must pass (``--skip-probes`` to skip);
5. serve - ``python -m oscar_b200.serve`` (under ``torch.distributed.run`` for more than
   one GPU) in its own process group, its output copied to ``--log``; a watcher collects
   the ranks' READY manifests, validates them (all ranks, one layer set, this source) and
   waits for ``/health``, then prints ``LAUNCH OK``.  A failed check, a serve process
   that exits first or ``--ready-timeout`` stops the server and the launch fails.

Arguments the launcher does not know are passed to the serve command.  The launcher stays
in the foreground until the server exits (``--exit-after-ready``: stop it once ready).
"""
from __future__ import annotations

import argparse
import os
import signal
import socket
import subprocess
import sys
import threading
import time
import urllib.request


def log(msg: str) -> None:
    print(f"[oscar-b200 launch] {msg}", flush=True)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def self_check(device: str | None) -> dict:
    from ..utils import platform as P

    info = P.collect()
    if device != "cpu":
        P.check_runtime(info)  # raises RuntimeMismatch
    log(f"self-check: torch {info['torch']}, {len(info['gpus'])} GPU(s), extension "
        f"{'loaded' if info['extension'].get('loaded') else 'not loaded'}")
    return info


def rotations(path: str, gpus: int, device: str | None, weights: str | None, model: str, calibrate: bool,
              layers: int | None) -> str | None:
    """Path of a v2 rotation checkpoint to serve with (None: seeded random rotations)."""
    import torch

    from ..kv.rotation import is_v2

    if os.path.exists(path):
        try:
            ok = is_v2(torch.load(path, map_location="cpu", weights_only=False))
        except Exception as e:  # noqa: BLE001 - an unreadable file is recalibrated
            log(f"rotations: {path} unreadable ({e!r})")
            ok = False
        if ok:
            log(f"rotations: reusing v2 checkpoint {path}")
            return path
        log(f"rotations: {path} is not a v2 checkpoint")
    if not calibrate:
        log("rotations: none, serving with seeded random rotations")
        return None
    cmd = _torchrun(gpus) + ["-m", "oscar_b200.kv.gen_rotations", "--out", path]
    cmd += ["--weights", weights] if weights else ["--model", model]
    if layers is not None:
        cmd += ["--layers", str(layers)]
    if device:
        cmd += ["--device", device]
    log(f"rotations: calibrating -> {path}")
    env = {**os.environ, "OSCAR_ASCEND_ENABLE": "0"}
    if subprocess.run(cmd, env=env).returncode != 0:
        raise RuntimeError("rotation calibration failed")
    return path


def _torchrun(gpus: int) -> list[str]:
    if gpus <= 1:
        return [sys.executable]
    return [sys.executable, "-m", "torch.distributed.run", "--nnodes", "1", "--nproc-per-node", str(gpus),
            "--master-addr", "127.0.0.1", "--master-port", str(_free_port())]


def _health(host: str, port: int) -> bool:
    try:
        with urllib.request.urlopen(f"http://{host}:{port}/health", timeout=2) as r:
            return r.status == 200
    except Exception:  # noqa: BLE001 - not up yet
        return False


def serve(args, extra: list[str], env: dict, sha: str) -> int:
    from ..engine.budget import BudgetError, parse_ready_lines, validate

    cmd = _torchrun(args.gpus) + ["-m", "oscar_b200.serve", "--host", args.host, "--port", str(args.port)] + extra
    log("serve: " + " ".join(cmd))
    logf = open(args.log, "w")
    proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, env=env, text=True,
                            start_new_session=True)
    lines: list[str] = []  # kept only until the READY check passed
    watching = threading.Event()
    watching.set()
    done = threading.Event()

    def pump():
        for ln in proc.stdout:
            logf.write(ln)
            logf.flush()
            sys.stdout.write(ln)
            if watching.is_set():
                lines.append(ln)
        done.set()

    threading.Thread(target=pump, daemon=True).start()

    def stop():
        if proc.poll() is None:
            os.killpg(proc.pid, signal.SIGTERM)  # the serve command's own process group
            try:
                proc.wait(60)
            except subprocess.TimeoutExpired:
                os.killpg(proc.pid, signal.SIGKILL)
                proc.wait()

    t0 = time.time()
    try:
        while True:
            if proc.poll() is not None:
                done.wait(10)
                log(f"FAILED: serve exited with {proc.returncode} before it was ready")
                return 1
            mans = parse_ready_lines("".join(lines))
            if len(mans) >= args.gpus:
                try:
                    validate(mans, world_size=args.gpus, sha256=sha)
                except BudgetError as e:
                    log(f"FAILED: READY check: {e}")
                    stop()
                    return 1
                if _health(args.host, args.port):
                    break
            if time.time() - t0 > args.ready_timeout:
                log(f"FAILED: not ready after {args.ready_timeout} s")
                stop()
                return 1
            time.sleep(0.2)
        watching.clear()
        lines.clear()
        log(f"LAUNCH OK: {len(mans)} rank(s), FULL layers {mans[0]['layer_ids']}, source {sha[:12]}, "
            f"http://{args.host}:{args.port}")
        if args.exit_after_ready:
            stop()
            return 0
        try:
            return proc.wait()
        except KeyboardInterrupt:
            stop()
            return 130
    finally:
        done.wait(10)
        logf.close()


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m oscar_b200.serve.launch")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--model", default="qwen35-27b")
    ap.add_argument("--weights", default=None)
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--device", default=None, help="cpu: the torch reference path (testing)")
    ap.add_argument("--rotations", default=None)
    ap.add_argument("--no-calibrate", action="store_true")
    ap.add_argument("--skip-probes", action="store_true")
    ap.add_argument("--log", default="serve.log")
    ap.add_argument("--ready-timeout", type=float, default=1800.0)
    ap.add_argument("--exit-after-ready", action="store_true")
    args, extra = ap.parse_known_args(argv)
    from ..engine.budget import source_fingerprint

    try:
        self_check(args.device)
    except Exception as e:  # noqa: BLE001
        log(f"FAILED: self-check: {e}")
        return 1
    sha = source_fingerprint()
    log(f"fingerprint: {sha}")
    env = dict(os.environ)
    path = args.rotations or os.environ.get("OSCAR_ASCEND_K_ROTATION_PATH") or "oscar_rotations.pt"
    try:
        rot = rotations(path, args.gpus, args.device, args.weights, args.model, not args.no_calibrate, args.layers)
    except RuntimeError as e:
        log(f"FAILED: {e}")
        return 1
    if rot:
        env["OSCAR_ASCEND_K_ROTATION_PATH"] = env["OSCAR_ASCEND_V_ROTATION_PATH"] = os.path.abspath(rot)
    if not args.skip_probes:
        log("probes: running")
        if subprocess.run([sys.executable, "-m", "oscar_b200.serve.probes"], env=env,
                          stdout=subprocess.DEVNULL).returncode != 0:
            log("FAILED: probes (run python -m oscar_b200.serve.probes for the report)")
            return 1
        log("probes: passed")
    passthrough = ["--model", args.model] + (["--weights", args.weights] if args.weights else [])
    passthrough += (["--layers", str(args.layers)] if args.layers is not None else [])
    passthrough += (["--device", args.device] if args.device else [])
    return serve(args, passthrough + extra, env, sha)


if __name__ == "__main__":
    sys.exit(main())
