"""The gym service: operations over the store, jobs in isolated worker processes, the HTTP API.

``GymService`` implements every operation of ``contract.OPERATIONS`` as a method taking the
validated parameters.  Work that runs model code (cost inspection, training) runs in a worker
subprocess (``gym.worker``) with a scrubbed environment, its own process group, resource limits
(CPU seconds, open files, core dumps off) and a wall-clock limit, so candidate code never runs in
the service process; a job slot runs one job at a time, GPU jobs wait for their lease.

``app(service, token)`` is the HTTP API: ``POST /v1/call`` with ``Authorization: Bearer <token>``
and ``{"schema_version", "operation", "params"}``; answers ``{"schema_version", "result"}`` or
``{"schema_version", "error": {"code", "message"}}`` with a matching HTTP status.
"""
import hmac
import json
import os
import queue
import resource
import signal
import subprocess
import sys
import threading
import time
import uuid
from pathlib import Path

from nexttransformer_b200.gym import contract
from nexttransformer_b200.gym.contract import GymError
from nexttransformer_b200.gym.package import candidate_from_package, unpack
from nexttransformer_b200.gym.resources import Leases, inventory
from nexttransformer_b200.gym.store import TERMINAL, Store

REPO = Path(__file__).resolve().parents[2]
_KEEP_ENV = ("PATH", "HOME", "LANG", "LC_ALL", "TMPDIR", "CUDA_HOME", "LD_LIBRARY_PATH", "NVIDIA_VISIBLE_DEVICES")


def _limits(cpu_seconds):
    def apply():
        os.setsid()
        resource.setrlimit(resource.RLIMIT_CPU, (cpu_seconds, cpu_seconds))
        resource.setrlimit(resource.RLIMIT_CORE, (0, 0))
        resource.setrlimit(resource.RLIMIT_NOFILE, (1024, 1024))
    return apply


class GymService:
    def __init__(self, state_dir, budget_flops, *, gpus=None, smi_runner=None, job_timeout=3600,
                 lease_ttl=600, python=sys.executable):
        self.root = Path(state_dir)
        self.root.mkdir(parents=True, exist_ok=True)
        self.store = Store(self.root / "gym.sqlite", budget_flops)
        self.leases = Leases(self.root / "leases.json")
        self.smi_runner, self.python = smi_runner, python
        self.job_timeout, self.lease_ttl = job_timeout, lease_ttl
        found = inventory(smi_runner)
        self.gpus = [g["index"] for g in found] if gpus is None else list(gpus)
        self._inventory = found
        self._queue = queue.Queue()
        self._procs, self._cancel = {}, set()
        self._lock = threading.Lock()
        self._worker = threading.Thread(target=self._run_jobs, name="gym-jobs", daemon=True)
        self._worker.start()

    # ------------------------------------------------------------------ dispatch
    def call(self, operation, params):
        params = contract.validate(operation, params)
        mutation = contract.OPERATIONS[operation]["mutation"]
        key = params.pop("idempotency_key", None) if mutation else None
        if key is not None:
            earlier = self.store.remembered(key, operation, params)
            if earlier is not None:
                return earlier
        result = getattr(self, "op_" + operation)(**params)
        if key is not None:
            self.store.remember(key, operation, params, result)
        return result

    # ------------------------------------------------------------------ operations
    def op_describe_space(self):
        return contract.describe()

    def op_get_resources(self):
        held = self.leases.held()
        return dict(gpus=[dict(g, leased=str(g["index"]) in held) for g in self._inventory if g["index"] in self.gpus],
                    allocated=self.gpus, free=self.leases.free(self.gpus), worker_slots=1)

    def op_submit_candidate(self, package_base64):
        cid, method, proposal, files = candidate_from_package(package_base64)
        path = self.root / "candidates" / cid
        if not path.exists():
            unpack(files, path)
        self.store.add_candidate(cid, method, proposal, path)
        self.store.event("candidate_submitted", candidate_id=cid, method=method)
        return dict(candidate_id=cid, method=method, files=sorted(files))

    def op_list_candidates(self, cursor, limit):
        items = self.store.candidates(cursor, limit)
        return dict(items=[{k: v for k, v in c.items() if k != "path"} for c in items],
                    next_cursor=items[-1]["candidate_id"] if len(items) == limit else None)

    def op_get_candidate(self, candidate_id):
        c = self.store.candidate(candidate_id)
        c["files"] = sorted(str(p.relative_to(c["path"])) for p in Path(c["path"]).rglob("*") if p.is_file())
        return {k: v for k, v in c.items() if k != "path"}

    def _profile(self, profile_id):
        if profile_id not in contract.PROFILES:
            raise GymError("not_found", f"no profile {profile_id}", 404)
        return contract.PROFILES[profile_id]

    def op_inspect_cost(self, candidate_id, profile_id):
        c = self.store.candidate(candidate_id)
        out = self._run_worker(dict(kind="cost", method=c["method"], profile=self._profile(profile_id)),
                               Path(c["path"]) / "plugin", gpus=[], timeout=600)
        if not out.get("ok"):
            raise GymError("candidate_failed", out.get("error", "cost inspection failed"), 422)
        return dict(candidate_id=candidate_id, profile_id=profile_id,
                    **{k: out[k] for k in ("parameters", "flops_per_token", "flops_per_update")})

    def op_quote_experiment(self, candidate_id, profile_id, target_update, gpus):
        cost = self.op_inspect_cost(candidate_id, profile_id)
        if gpus > len(self.gpus):
            raise GymError("resources", f"{gpus} GPUs requested, {len(self.gpus)} allocated to this gym")
        qid = "quote_" + uuid.uuid4().hex[:16]
        body = dict(quote_id=qid, candidate_id=candidate_id, profile_id=profile_id, target_update=target_update,
                    gpus=gpus, flops=cost["flops_per_update"] * target_update)
        body["affordable"] = body["flops"] <= self.store.budget()["available"]
        self.store.put("quotes", qid, body)
        return body

    def op_run_experiment(self, quote_id):
        q = self.store.get("quotes", quote_id)
        jid = "job_" + uuid.uuid4().hex[:16]
        self.store.open_job(jid, quote_id, q["flops"])
        self.store.event("job_queued", job_id=jid, quote_id=quote_id, flops=q["flops"])
        self._queue.put(jid)
        return self.store.job(jid)

    def op_get_job(self, job_id):
        return self.store.job(job_id)

    def op_get_result(self, job_id):
        j = self.store.job(job_id)
        if j["state"] not in TERMINAL:
            raise GymError("not_ready", f"job {job_id} is {j['state']}", 409)
        return dict(job_id=job_id, state=j["state"], result=j["result"], spent_flops=j["spent_flops"])

    def op_cancel_job(self, job_id):
        j = self.store.job(job_id)
        if j["state"] in TERMINAL:
            return j
        with self._lock:
            self._cancel.add(job_id)
            proc = self._procs.get(job_id)
        if proc is not None:
            try:
                os.killpg(proc.pid, signal.SIGTERM)
            except ProcessLookupError:
                pass
        if j["state"] == "queued":
            self.store.close_job(job_id, "cancelled", 0.0)
            self.store.event("job_cancelled", job_id=job_id)
        return self.store.job(job_id)

    def op_read_events(self, cursor, limit):
        items = self.store.events(cursor, limit)
        return dict(items=items, next_cursor=items[-1]["seq"] if items else cursor)

    def op_get_budget(self):
        return self.store.budget()

    def op_finalize(self, candidate_id, profile_id):
        self.store.candidate(candidate_id)
        self._profile(profile_id)
        sid = "sub_" + uuid.uuid4().hex[:16]
        body = dict(submission_id=sid, candidate_id=candidate_id, profile_id=profile_id, frozen_at=time.time())
        self.store.put("submissions", sid, body)
        self.store.event("finalized", **body)
        return body

    def op_get_submission(self, submission_id):
        return self.store.get("submissions", submission_id)

    # ------------------------------------------------------------------ jobs
    def _run_worker(self, job, plugin_root, gpus, timeout, job_id=None):
        work = self.root / "work" / (job_id or uuid.uuid4().hex[:16])
        work.mkdir(parents=True, exist_ok=True)
        (work / "job.json").write_text(json.dumps(job))
        env = {k: os.environ[k] for k in _KEEP_ENV if k in os.environ}
        env.update(NEXTTRANSFORMER_METHOD_PATHS=str(plugin_root), PYTHONPATH=str(REPO),
                   CUDA_VISIBLE_DEVICES=",".join(str(g) for g in gpus), PYTHONDONTWRITEBYTECODE="1")
        proc = subprocess.Popen([self.python, "-m", "nexttransformer_b200.gym.worker", str(work / "job.json")],
                                cwd=work, env=env, stdout=open(work / "stdout.log", "w"),
                                stderr=subprocess.STDOUT, preexec_fn=_limits(int(timeout) + 60))
        if job_id is not None:
            with self._lock:
                self._procs[job_id] = proc
        try:
            proc.wait(timeout=timeout)
        except subprocess.TimeoutExpired:
            os.killpg(proc.pid, signal.SIGKILL)
            proc.wait()
            return dict(ok=False, error=f"time limit of {timeout} s reached")
        finally:
            if job_id is not None:
                with self._lock:
                    self._procs.pop(job_id, None)
        path = work / "result.json"
        if not path.exists():
            return dict(ok=False, error=f"worker exited with code {proc.returncode}")
        return json.loads(path.read_text())

    def _run_jobs(self):
        while True:
            jid = self._queue.get()
            if jid is None:
                return
            try:
                self._run_one(jid)
            except Exception as e:  # the job fails, the service keeps serving
                self.store.close_job(jid, "failed", 0.0, dict(error=f"{type(e).__name__}: {e}"))

    def _run_one(self, jid):
        job = self.store.job(jid)
        if job["state"] in TERMINAL:
            return
        q = self.store.get("quotes", job["quote_id"])
        c = self.store.candidate(q["candidate_id"])
        gpus = []
        if q["gpus"]:
            while True:
                free = self.leases.free(self.gpus)
                if len(free) >= q["gpus"] and self.leases.acquire(free[:q["gpus"]], jid, self.lease_ttl):
                    gpus = free[:q["gpus"]]
                    break
                with self._lock:
                    if jid in self._cancel:
                        return
                time.sleep(1.0)
        self.store.set_state(jid, "running", dict(gpus=gpus))
        self.store.event("job_started", job_id=jid, gpus=gpus)
        try:
            out = self._run_worker(dict(kind="train", method=c["method"], profile=self._profile(q["profile_id"]),
                                        target_update=q["target_update"]),
                                   Path(c["path"]) / "plugin", gpus, self.job_timeout, job_id=jid)
        finally:
            if gpus:
                self.leases.release(jid)
        with self._lock:
            cancelled = jid in self._cancel
        if cancelled:
            state = "cancelled"
        else:
            state = "succeeded" if out.get("ok") else "failed"
        used = out.get("flops", 0.0) if out.get("ok") else 0.0
        self.store.close_job(jid, state, used, out)
        self.store.event("job_" + state, job_id=jid, spent_flops=used)

    def close(self):
        self._queue.put(None)


def app(service, token):
    """FastAPI application of ``service`` guarded by a bearer ``token``."""
    from fastapi import FastAPI, Request
    from fastapi.responses import JSONResponse
    api = FastAPI(title="nexttransformer_b200 gym", version=contract.SCHEMA_VERSION)

    def answer(status, **body):
        return JSONResponse(status_code=status, content=dict(schema_version=contract.SCHEMA_VERSION, **body))

    @api.get("/v1/health")
    def health():
        return {"ok": True}

    @api.post("/v1/call")
    async def call(request: Request):
        auth = request.headers.get("authorization", "")
        if not hmac.compare_digest(auth.encode(), f"Bearer {token}".encode()):
            return answer(401, error=dict(code="unauthorized", message="missing or wrong bearer token"))
        try:
            body = await request.json()
        except ValueError:
            return answer(400, error=dict(code="invalid_json", message="request body is not JSON"))
        if not isinstance(body, dict) or body.get("schema_version") != contract.SCHEMA_VERSION:
            return answer(400, error=dict(code="schema_version", message=f"expected {contract.SCHEMA_VERSION}"))
        try:
            import anyio
            result = await anyio.to_thread.run_sync(service.call, body.get("operation"), body.get("params") or {})
        except GymError as e:
            return answer(e.status, error=dict(code=e.code, message=e.message))
        return answer(200, result=result)

    return api
