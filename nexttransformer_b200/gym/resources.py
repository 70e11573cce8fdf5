"""GPUs of the host and exclusive leases on them.

``inventory`` reads ``nvidia-smi -q -x`` (the runner is injectable, so tests feed recorded XML):
index, UUID, name, memory and the number of running compute processes per GPU.  ``Leases`` hands
out whole GPU groups all-or-nothing from a JSON file under an ``fcntl`` lock, so several gym
processes on one host share one view; a lease carries its owner and expiry, and an expired lease
is reclaimed on the next acquisition.  A busy GPU keeps a job waiting: a job never falls back to
another device kind.
"""
import fcntl
import json
import subprocess
import time
import xml.etree.ElementTree as ET
from pathlib import Path


def _mib(text):
    try:
        return int(str(text).split()[0])
    except (ValueError, IndexError, AttributeError):
        return None


def parse_nvidia_smi(xml_text):
    """[{index, uuid, name, memory_total_mib, memory_used_mib, processes}] from ``nvidia-smi -q -x``."""
    root = ET.fromstring(xml_text)
    gpus = []
    for i, gpu in enumerate(root.findall("gpu")):
        mem = gpu.find("fb_memory_usage")
        procs = gpu.find("processes")
        gpus.append(dict(
            index=int(gpu.findtext("minor_number", str(i)) or i), uuid=gpu.findtext("uuid", ""),
            name=gpu.findtext("product_name", ""),
            memory_total_mib=_mib(mem.findtext("total")) if mem is not None else None,
            memory_used_mib=_mib(mem.findtext("used")) if mem is not None else None,
            processes=len(procs.findall("process_info")) if procs is not None else 0))
    return gpus


def inventory(runner=None):
    """The host's GPUs ([] without a driver)."""
    def run():
        return subprocess.run(["nvidia-smi", "-q", "-x"], capture_output=True, text=True, timeout=30,
                              check=True).stdout
    try:
        return parse_nvidia_smi((runner or run)())
    except (OSError, subprocess.SubprocessError, ET.ParseError):
        return []


class Leases:
    def __init__(self, path, clock=time.time):
        self.path, self.clock = Path(path), clock
        self.path.parent.mkdir(parents=True, exist_ok=True)
        self.path.touch(exist_ok=True)

    def _locked(self, fn):
        with open(self.path, "r+") as f:
            fcntl.flock(f, fcntl.LOCK_EX)
            try:
                text = f.read()
                table = json.loads(text) if text.strip() else {}
                now = self.clock()
                table = {g: lease for g, lease in table.items() if lease["expires"] > now}
                out = fn(table, now)
                f.seek(0)
                f.truncate()
                f.write(json.dumps(table))
                return out
            finally:
                fcntl.flock(f, fcntl.LOCK_UN)

    def acquire(self, gpus, owner, ttl):
        """Lease every GPU of ``gpus`` to ``owner`` for ``ttl`` seconds, or none of them; returns success."""
        keys = [str(g) for g in gpus]

        def take(table, now):
            if any(k in table and table[k]["owner"] != owner for k in keys):
                return False
            for k in keys:
                table[k] = dict(owner=owner, expires=now + ttl)
            return True
        return self._locked(take)

    def renew(self, owner, ttl):
        def ren(table, now):
            for lease in table.values():
                if lease["owner"] == owner:
                    lease["expires"] = now + ttl
        self._locked(ren)

    def release(self, owner):
        def rel(table, now):
            for k in [k for k, lease in table.items() if lease["owner"] == owner]:
                del table[k]
        self._locked(rel)

    def held(self):
        return self._locked(lambda table, now: {k: dict(v) for k, v in table.items()})

    def free(self, gpus):
        held = self.held()
        return [g for g in gpus if str(g) not in held]
