"""Gym entry points.

    python -m nexttransformer_b200.gym serve --state DIR --budget-flops 1e18 [--port 8765] [--gpus 0 1]
    python -m nexttransformer_b200.gym mcp --credential credential.json

``serve`` writes ``<state>/credential.json`` (endpoint and a fresh bearer token, mode 0600) for the
client and the MCP adapter, and serves the HTTP API on 127.0.0.1.
"""
import argparse
import json
import os
import secrets
from pathlib import Path


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="cmd", required=True)
    s = sub.add_parser("serve")
    s.add_argument("--state", type=Path, required=True)
    s.add_argument("--budget-flops", type=float, required=True)
    s.add_argument("--port", type=int, default=8765)
    s.add_argument("--gpus", type=int, nargs="*")
    s.add_argument("--job-timeout", type=int, default=3600)
    m = sub.add_parser("mcp")
    m.add_argument("--credential", type=Path, required=True)
    a = ap.parse_args(argv)
    if a.cmd == "serve":
        import uvicorn
        from nexttransformer_b200.gym.service import GymService, app
        service = GymService(a.state, a.budget_flops, gpus=a.gpus, job_timeout=a.job_timeout)
        token = secrets.token_urlsafe(32)
        cred = a.state / "credential.json"
        cred.write_text(json.dumps(dict(endpoint=f"http://127.0.0.1:{a.port}", token=token)))
        os.chmod(cred, 0o600)
        uvicorn.run(app(service, token), host="127.0.0.1", port=a.port, log_level="warning")
    else:
        from nexttransformer_b200.gym.client import GymClient
        from nexttransformer_b200.gym.mcp import serve
        client = GymClient.from_credential(a.credential)
        serve(lambda op, params: client.call(op, **params))


if __name__ == "__main__":
    main()
