"""Durable gym state in one SQLite file: candidates, quotes, jobs, events, the FLOP budget,
submissions and idempotency keys.

Budget accounting: ``run_experiment`` moves a quote's FLOPs from available to reserved in one
transaction (refused when they do not fit); a finished job moves what it used to spent and gives
the rest back; a cancelled or failed job gives back what it did not use.  Mutations carrying an
idempotency key return the first call's result when repeated with the same input, and are refused
when the key comes back with different input.
"""
import hashlib
import json
import sqlite3
import threading
import time

from nexttransformer_b200.gym.contract import GymError

_SCHEMA = """
CREATE TABLE IF NOT EXISTS candidates (id TEXT PRIMARY KEY, method TEXT, proposal TEXT, path TEXT, created REAL);
CREATE TABLE IF NOT EXISTS quotes (id TEXT PRIMARY KEY, body TEXT, created REAL);
CREATE TABLE IF NOT EXISTS jobs (id TEXT PRIMARY KEY, quote TEXT, state TEXT, reserved REAL, spent REAL,
                                 progress TEXT, result TEXT, created REAL, updated REAL);
CREATE TABLE IF NOT EXISTS events (seq INTEGER PRIMARY KEY AUTOINCREMENT, at REAL, kind TEXT, body TEXT);
CREATE TABLE IF NOT EXISTS budget (id INTEGER PRIMARY KEY CHECK (id = 0), limit_flops REAL, spent REAL, reserved REAL);
CREATE TABLE IF NOT EXISTS submissions (id TEXT PRIMARY KEY, body TEXT, created REAL);
CREATE TABLE IF NOT EXISTS idempotency (key TEXT PRIMARY KEY, op TEXT, digest TEXT, result TEXT);
"""
TERMINAL = ("succeeded", "failed", "cancelled")


def _digest(op, params):
    return hashlib.sha256(json.dumps([op, params], sort_keys=True).encode()).hexdigest()


class Store:
    def __init__(self, path, budget_flops):
        self._db = sqlite3.connect(str(path), check_same_thread=False, isolation_level=None)
        self._lock = threading.RLock()
        with self._lock:
            self._db.executescript(_SCHEMA)
            self._db.execute("INSERT OR IGNORE INTO budget VALUES (0, ?, 0, 0)", (float(budget_flops),))

    def _tx(self):
        store = self

        class _T:
            def __enter__(self):
                store._lock.acquire()
                store._db.execute("BEGIN IMMEDIATE")
                return store._db

            def __exit__(self, kind, *_):
                store._db.execute("ROLLBACK" if kind else "COMMIT")
                store._lock.release()
        return _T()

    # ------------------------------------------------------------------ idempotency
    def remembered(self, key, op, params):
        """The stored result of an earlier call with this key, or None."""
        if not key:
            return None
        with self._lock:
            row = self._db.execute("SELECT op, digest, result FROM idempotency WHERE key = ?", (key,)).fetchone()
        if row is None:
            return None
        if row[0] != op or row[1] != _digest(op, params):
            raise GymError("idempotency_conflict", "idempotency key reused with different input", 409)
        return json.loads(row[2])

    def remember(self, key, op, params, result):
        if key:
            with self._lock:
                self._db.execute("INSERT OR IGNORE INTO idempotency VALUES (?, ?, ?, ?)",
                                 (key, op, _digest(op, params), json.dumps(result)))

    # ------------------------------------------------------------------ events
    def event(self, kind, **body):
        with self._lock:
            self._db.execute("INSERT INTO events (at, kind, body) VALUES (?, ?, ?)", (time.time(), kind,
                                                                                    json.dumps(body)))

    def events(self, cursor, limit):
        with self._lock:
            rows = self._db.execute("SELECT seq, at, kind, body FROM events WHERE seq > ? ORDER BY seq LIMIT ?",
                                    (cursor, limit)).fetchall()
        return [dict(seq=s, at=a, kind=k, **json.loads(b)) for s, a, k, b in rows]

    # ------------------------------------------------------------------ candidates, quotes, submissions
    def add_candidate(self, cid, method, proposal, path):
        with self._lock:
            self._db.execute("INSERT OR IGNORE INTO candidates VALUES (?, ?, ?, ?, ?)",
                             (cid, method, json.dumps(proposal), str(path), time.time()))

    def candidate(self, cid):
        with self._lock:
            row = self._db.execute("SELECT id, method, proposal, path, created FROM candidates WHERE id = ?",
                                   (cid,)).fetchone()
        if row is None:
            raise GymError("not_found", f"no candidate {cid}", 404)
        return dict(candidate_id=row[0], method=row[1], proposal=json.loads(row[2]), path=row[3], created=row[4])

    def candidates(self, after, limit):
        with self._lock:
            rows = self._db.execute("SELECT id FROM candidates WHERE id > ? ORDER BY id LIMIT ?",
                                    (after, limit)).fetchall()
        return [self.candidate(r[0]) for r in rows]

    def put(self, table, key, body):
        with self._lock:
            self._db.execute(f"INSERT INTO {table} VALUES (?, ?, ?)", (key, json.dumps(body), time.time()))

    def get(self, table, key):
        with self._lock:
            row = self._db.execute(f"SELECT body FROM {table} WHERE id = ?", (key,)).fetchone()
        if row is None:
            raise GymError("not_found", f"no {table[:-1]} {key}", 404)
        return json.loads(row[0])

    # ------------------------------------------------------------------ budget and jobs
    def budget(self):
        with self._lock:
            limit, spent, reserved = self._db.execute("SELECT limit_flops, spent, reserved FROM budget").fetchone()
        return dict(limit=limit, spent=spent, reserved=reserved, available=limit - spent - reserved)

    def open_job(self, job_id, quote_id, flops):
        """Reserve ``flops`` and create the job in one transaction."""
        with self._tx() as db:
            limit, spent, reserved = db.execute("SELECT limit_flops, spent, reserved FROM budget").fetchone()
            if flops > limit - spent - reserved:
                raise GymError("budget_exceeded", f"{flops:.3e} FLOPs requested, {limit - spent - reserved:.3e} "
                                                  "available", 402)
            db.execute("UPDATE budget SET reserved = reserved + ?", (flops,))
            now = time.time()
            db.execute("INSERT INTO jobs VALUES (?, ?, 'queued', ?, 0, '{}', NULL, ?, ?)",
                       (job_id, quote_id, flops, now, now))

    def job(self, job_id):
        with self._lock:
            row = self._db.execute("SELECT id, quote, state, reserved, spent, progress, result, created, updated "
                                   "FROM jobs WHERE id = ?", (job_id,)).fetchone()
        if row is None:
            raise GymError("not_found", f"no job {job_id}", 404)
        return dict(job_id=row[0], quote_id=row[1], state=row[2], reserved_flops=row[3], spent_flops=row[4],
                    progress=json.loads(row[5]), result=json.loads(row[6]) if row[6] else None, created=row[7],
                    updated=row[8])

    def set_state(self, job_id, state, progress=None):
        with self._lock:
            self._db.execute("UPDATE jobs SET state = ?, progress = COALESCE(?, progress), updated = ? WHERE id = ?",
                             (state, json.dumps(progress) if progress is not None else None, time.time(), job_id))

    def close_job(self, job_id, state, used_flops, result=None):
        """Settle a job's reservation: ``used_flops`` (at most the reservation) become spent."""
        if state not in TERMINAL:
            raise ValueError(state)
        with self._tx() as db:
            reserved, old = db.execute("SELECT reserved, state FROM jobs WHERE id = ?", (job_id,)).fetchone()
            if old in TERMINAL:
                return
            used = min(max(float(used_flops), 0.0), reserved)
            db.execute("UPDATE budget SET reserved = reserved - ?, spent = spent + ?", (reserved, used))
            db.execute("UPDATE jobs SET state = ?, spent = ?, reserved = 0, result = ?, updated = ? WHERE id = ?",
                       (state, used, json.dumps(result) if result is not None else None, time.time(), job_id))
