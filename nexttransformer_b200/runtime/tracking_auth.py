"""W&B login checked before any process group exists (``nexttransformer/runtime/tracking_auth.py``
of the reference): a missing or wrong credential must fail in seconds on rank zero, not after every
rank has joined NCCL.  The check runs in a bounded, non-interactive child process whose output is
never echoed (SDK messages can contain secrets); its exit code names the failure.
"""
import subprocess
import sys

# exit code of the child -> reason
REASONS = {2: "no W&B API key is configured in this training container",
           3: "W&B credentials could not be verified (credentials or network)",
           4: "W&B is not installed in this environment"}


def preflight(mode, timeout=60, runner=subprocess.run):
    if mode != "online":
        return
    try:
        result = runner([sys.executable, "-m", "nexttransformer_b200.runtime.tracking_auth"],
                        stdin=subprocess.DEVNULL, stdout=subprocess.PIPE, stderr=subprocess.PIPE, timeout=timeout,
                        check=False)
    except subprocess.TimeoutExpired:
        raise RuntimeError(f"W&B authentication timed out after {timeout}s; check access to the W&B server") from None
    if result.returncode:
        reason = REASONS.get(result.returncode, "the W&B authentication check failed")
        raise RuntimeError(reason + "; provide WANDB_API_KEY or a netrc file in the container")
    print("W&B online authentication verified before distributed initialization.", flush=True)


def _verify():
    try:
        import wandb
    except ImportError:
        return 4
    try:
        return 0 if wandb.login(verify=True, prompt=False) else 2
    except Exception:
        return 3


if __name__ == "__main__":
    raise SystemExit(_verify())
