"""Account ledger service: accounts with token allocations, API keys with per-key caps,
and a no-overshoot reserve -> settle ledger that gateways call before and after
every request (the reference's crates/helexa-upstream: ledger.rs, authz.rs, topup.rs,
web.rs, on Postgres).

Storage is SQLite. Every ledger mutation runs in one `BEGIN IMMEDIATE` transaction,
which takes the database's write lock before reading the balances it checks, so two
concurrent reservations can never both pass a check that only one of them fits (the
reference gets the same guarantee from `SELECT ... FOR UPDATE` row locks).

Ledger rules:
* available = min(account total - spent - reserved, key cap - key spent - key reserved),
  key cap = `hardcap` value, or `percent` of the account total;
* reserve(max_tokens) fails with insufficient_quota when max_tokens > available,
  otherwise records an open reservation and adds it to both reserved counters;
* settle(actual) charges min(max(actual, 0), reserved) and releases the reservation;
  release() returns it unspent; both are idempotent (a closed reservation is a no-op);
* open reservations older than `stale_s` are released by the sweeper.

HTTP:
  /authz/v1/{resolve,reserve,settle,release,snapshot,served-usage}  (operator bearer tokens)
  /web/v1/{register,login,account,keys,keys/{id}/archive,allocation,redeem}  (session tokens)
  /health
"""
from __future__ import annotations

import hashlib
import hmac
import secrets
import sqlite3
import threading
import time
import uuid
from dataclasses import dataclass, field

from fastapi import FastAPI, Request
from fastapi.responses import JSONResponse

SCHEMA = """
CREATE TABLE IF NOT EXISTS accounts (
  id TEXT PRIMARY KEY, email TEXT UNIQUE, pw_hash BLOB, pw_salt BLOB, status TEXT NOT NULL DEFAULT 'active',
  allocation_total INTEGER NOT NULL DEFAULT 0, allocation_spent INTEGER NOT NULL DEFAULT 0,
  allocation_reserved INTEGER NOT NULL DEFAULT 0, created_at REAL NOT NULL);
CREATE TABLE IF NOT EXISTS api_keys (
  id TEXT PRIMARY KEY, account_id TEXT NOT NULL REFERENCES accounts(id), key_hash BLOB UNIQUE NOT NULL,
  label TEXT, status TEXT NOT NULL DEFAULT 'active', limit_kind TEXT NOT NULL DEFAULT 'percent',
  limit_value INTEGER NOT NULL DEFAULT 100, key_spent INTEGER NOT NULL DEFAULT 0,
  key_reserved INTEGER NOT NULL DEFAULT 0, created_at REAL NOT NULL);
CREATE TABLE IF NOT EXISTS reservations (
  id INTEGER PRIMARY KEY AUTOINCREMENT, account_id TEXT NOT NULL, key_id TEXT NOT NULL, reserved INTEGER NOT NULL,
  actual INTEGER, state TEXT NOT NULL, created_at REAL NOT NULL, settled_at REAL);
CREATE TABLE IF NOT EXISTS topup_codes (
  code_hash BLOB PRIMARY KEY, tokens INTEGER NOT NULL, redeemed_by TEXT, redeemed_at REAL);
CREATE TABLE IF NOT EXISTS served_usage (
  id INTEGER PRIMARY KEY AUTOINCREMENT, operator TEXT, model TEXT, prompt_tokens INTEGER,
  completion_tokens INTEGER, at REAL);
CREATE TABLE IF NOT EXISTS sessions (token_hash BLOB PRIMARY KEY, account_id TEXT NOT NULL, expires REAL NOT NULL);
"""


def sha256(s: str) -> bytes:
    return hashlib.sha256(s.encode()).digest()


def resolve_abs_cap(limit_kind: str, limit_value: int, allocation_total: int) -> int:
    cap = allocation_total * limit_value // 100 if limit_kind == "percent" else limit_value
    return max(0, cap)


class LedgerError(Exception):
    code = "ledger_error"
    status = 400


class NotFound(LedgerError):
    code = "not_found"
    status = 404


class InsufficientQuota(LedgerError):
    code = "insufficient_quota"
    status = 402

    def __init__(self, requested: int, available: int):
        super().__init__(f"insufficient quota: requested {requested}, available {available}")
        self.requested, self.available = requested, available


class Ledger:
    def __init__(self, path: str = ":memory:"):
        self.db = sqlite3.connect(path, check_same_thread=False, isolation_level=None)
        self.db.row_factory = sqlite3.Row
        self.db.executescript(SCHEMA)
        self._lock = threading.Lock()  # one connection: serialise its use across threads

    def _tx(self):
        ledger = self

        class _T:
            def __enter__(self):
                ledger._lock.acquire()
                ledger.db.execute("BEGIN IMMEDIATE")
                return ledger.db

            def __exit__(self, et, e, tb):
                try:
                    ledger.db.execute("ROLLBACK" if et else "COMMIT")
                finally:
                    ledger._lock.release()
        return _T()

    # ---- accounts and keys ----
    def create_account(self, email: str | None = None, allocation: int = 0, password: str | None = None) -> str:
        aid = str(uuid.uuid4())
        salt = secrets.token_bytes(16)
        pw = hashlib.scrypt(password.encode(), salt=salt, n=2**14, r=8, p=1) if password else None
        with self._tx() as db:
            db.execute("INSERT INTO accounts (id, email, pw_hash, pw_salt, allocation_total, created_at) "
                       "VALUES (?, ?, ?, ?, ?, ?)", (aid, email, pw, salt, allocation, time.time()))
        return aid

    def check_password(self, email: str, password: str) -> str | None:
        r = self.db.execute("SELECT id, pw_hash, pw_salt FROM accounts WHERE email = ? AND status = 'active'",
                            (email,)).fetchone()
        if r is None or r["pw_hash"] is None:
            return None
        h = hashlib.scrypt(password.encode(), salt=r["pw_salt"], n=2**14, r=8, p=1)
        return r["id"] if hmac.compare_digest(h, r["pw_hash"]) else None

    def create_key(self, account_id: str, label: str = "", limit_kind: str = "percent",
                   limit_value: int = 100) -> tuple[str, str]:
        if limit_kind not in ("percent", "hardcap") or limit_value < 0:
            raise LedgerError("limit_kind must be percent or hardcap with a non-negative value")
        raw = "hx-" + secrets.token_urlsafe(32)
        kid = str(uuid.uuid4())
        with self._tx() as db:
            if db.execute("SELECT 1 FROM accounts WHERE id = ?", (account_id,)).fetchone() is None:
                raise NotFound("account not found")
            db.execute("INSERT INTO api_keys (id, account_id, key_hash, label, limit_kind, limit_value, created_at) "
                       "VALUES (?, ?, ?, ?, ?, ?, ?)", (kid, account_id, sha256(raw), label, limit_kind, limit_value,
                                                        time.time()))
        return kid, raw

    def archive_key(self, account_id: str, key_id: str) -> bool:
        with self._tx() as db:
            n = db.execute("UPDATE api_keys SET status = 'archived' WHERE id = ? AND account_id = ?",
                           (key_id, account_id)).rowcount
        return n > 0

    def list_keys(self, account_id: str) -> list[dict]:
        rows = self.db.execute("SELECT id, label, status, limit_kind, limit_value, key_spent, key_reserved "
                               "FROM api_keys WHERE account_id = ? ORDER BY created_at", (account_id,)).fetchall()
        return [dict(r) for r in rows]

    def account(self, account_id: str) -> dict:
        r = self.db.execute("SELECT id, email, status, allocation_total, allocation_spent, allocation_reserved "
                            "FROM accounts WHERE id = ?", (account_id,)).fetchone()
        if r is None:
            raise NotFound("account not found")
        return dict(r)

    # ---- ledger ----
    def resolve_key(self, api_key: str) -> dict | None:
        r = self.db.execute(
            "SELECT k.id AS key_id, k.account_id, k.limit_kind, k.limit_value, k.key_spent, k.key_reserved, "
            "a.allocation_total FROM api_keys k JOIN accounts a ON a.id = k.account_id "
            "WHERE k.key_hash = ? AND k.status = 'active' AND a.status = 'active'", (sha256(api_key),)).fetchone()
        if r is None:
            return None
        return {"account_id": r["account_id"], "key_id": r["key_id"],
                "hard_cap": resolve_abs_cap(r["limit_kind"], r["limit_value"], r["allocation_total"]),
                "spent": r["key_spent"], "reserved": r["key_reserved"]}

    def snapshot(self, account_id: str, key_id: str) -> dict:
        r = self.db.execute(
            "SELECT k.limit_kind, k.limit_value, k.key_spent, k.key_reserved, a.allocation_total "
            "FROM api_keys k JOIN accounts a ON a.id = k.account_id WHERE k.id = ? AND k.account_id = ? "
            "AND k.status = 'active' AND a.status = 'active'", (key_id, account_id)).fetchone()
        if r is None:
            raise NotFound("api key not found or not active")
        return {"hard_cap": resolve_abs_cap(r["limit_kind"], r["limit_value"], r["allocation_total"]),
                "spent": r["key_spent"], "reserved": r["key_reserved"]}

    def reserve(self, account_id: str, key_id: str, max_tokens: int) -> int:
        if max_tokens < 0:
            raise LedgerError("max_tokens must be non-negative")
        with self._tx() as db:
            a = db.execute("SELECT allocation_total, allocation_spent, allocation_reserved FROM accounts "
                           "WHERE id = ? AND status = 'active'", (account_id,)).fetchone()
            if a is None:
                raise NotFound("account not found")
            k = db.execute("SELECT limit_kind, limit_value, key_spent, key_reserved FROM api_keys "
                           "WHERE id = ? AND account_id = ? AND status = 'active'", (key_id, account_id)).fetchone()
            if k is None:
                raise NotFound("api key not found or not active")
            acct_avail = a["allocation_total"] - a["allocation_spent"] - a["allocation_reserved"]
            key_avail = resolve_abs_cap(k["limit_kind"], k["limit_value"], a["allocation_total"]) \
                - k["key_spent"] - k["key_reserved"]
            available = max(0, min(acct_avail, key_avail))
            if max_tokens > available:
                raise InsufficientQuota(max_tokens, available)
            rid = db.execute("INSERT INTO reservations (account_id, key_id, reserved, state, created_at) "
                             "VALUES (?, ?, ?, 'open', ?)", (account_id, key_id, max_tokens, time.time())).lastrowid
            db.execute("UPDATE accounts SET allocation_reserved = allocation_reserved + ? WHERE id = ?",
                       (max_tokens, account_id))
            db.execute("UPDATE api_keys SET key_reserved = key_reserved + ? WHERE id = ?", (max_tokens, key_id))
        return rid

    def _close(self, rid: int, actual: int | None):
        with self._tx() as db:
            r = db.execute("SELECT account_id, key_id, reserved FROM reservations WHERE id = ? AND state = 'open'",
                           (rid,)).fetchone()
            if r is None:
                return  # unknown or already closed: idempotent
            charged = 0 if actual is None else min(max(actual, 0), r["reserved"])
            db.execute("UPDATE reservations SET state = ?, actual = ?, settled_at = ? WHERE id = ?",
                       ("released" if actual is None else "settled", charged, time.time(), rid))
            db.execute("UPDATE accounts SET allocation_reserved = allocation_reserved - ?, "
                       "allocation_spent = allocation_spent + ? WHERE id = ?", (r["reserved"], charged, r["account_id"]))
            db.execute("UPDATE api_keys SET key_reserved = key_reserved - ?, key_spent = key_spent + ? WHERE id = ?",
                       (r["reserved"], charged, r["key_id"]))

    def settle(self, rid: int, actual_tokens: int):
        self._close(rid, int(actual_tokens))

    def release(self, rid: int):
        self._close(rid, None)

    def sweep_stale(self, max_age_s: float) -> int:
        old = self.db.execute("SELECT id FROM reservations WHERE state = 'open' AND created_at < ?",
                              (time.time() - max_age_s,)).fetchall()
        for r in old:
            self.release(r["id"])
        return len(old)

    def record_served(self, operator: str, model: str, prompt: int, completion: int):
        with self._tx() as db:
            db.execute("INSERT INTO served_usage (operator, model, prompt_tokens, completion_tokens, at) "
                       "VALUES (?, ?, ?, ?, ?)", (operator, model, prompt, completion, time.time()))

    # ---- top-up codes ----
    def mint_code(self, tokens: int) -> str:
        raw = "TOP-" + secrets.token_hex(8).upper()
        with self._tx() as db:
            db.execute("INSERT INTO topup_codes (code_hash, tokens) VALUES (?, ?)", (sha256(raw), tokens))
        return raw

    def redeem(self, account_id: str, raw_code: str) -> int:
        with self._tx() as db:
            r = db.execute("SELECT tokens, redeemed_by FROM topup_codes WHERE code_hash = ?",
                           (sha256(raw_code.strip()),)).fetchone()
            if r is None or r["redeemed_by"] is not None:
                raise LedgerError("code is invalid or already redeemed")
            db.execute("UPDATE topup_codes SET redeemed_by = ?, redeemed_at = ? WHERE code_hash = ?",
                       (account_id, time.time(), sha256(raw_code.strip())))
            db.execute("UPDATE accounts SET allocation_total = allocation_total + ? WHERE id = ?",
                       (r["tokens"], account_id))
        return r["tokens"]

    # ---- sessions ----
    def new_session(self, account_id: str, ttl_s: float = 86400.0) -> str:
        tok = secrets.token_urlsafe(32)
        with self._tx() as db:
            db.execute("INSERT INTO sessions (token_hash, account_id, expires) VALUES (?, ?, ?)",
                       (sha256(tok), account_id, time.time() + ttl_s))
        return tok

    def session_account(self, tok: str) -> str | None:
        r = self.db.execute("SELECT account_id, expires FROM sessions WHERE token_hash = ?", (sha256(tok),)).fetchone()
        return r["account_id"] if r is not None and r["expires"] > time.time() else None


@dataclass
class UpstreamConfig:
    db_path: str = ":memory:"
    operator_tokens: dict = field(default_factory=dict)   # token -> operator id (empty: open, dev only)
    signup_allocation: int = 0
    stale_reservation_s: float = 900.0


def _err(status: int, msg: str, code: str):
    return JSONResponse({"error": {"message": msg, "type": "invalid_request_error", "code": code}}, status_code=status)


def create_upstream(cfg: UpstreamConfig | None = None, ledger: Ledger | None = None) -> FastAPI:
    cfg = cfg or UpstreamConfig()
    L = ledger or Ledger(cfg.db_path)
    app = FastAPI(title="helexa-b200 upstream ledger")
    app.state.ledger = L

    def bearer(req: Request) -> str:
        h = req.headers.get("authorization", "")
        return h[7:].strip() if h.startswith("Bearer ") else ""

    def operator(req: Request) -> str | None:
        if not cfg.operator_tokens:
            return "dev"
        tok = bearer(req)
        for t, op in cfg.operator_tokens.items():
            if hmac.compare_digest(t.encode(), tok.encode()):
                return op
        return None

    async def authz(req: Request, fn):
        op = operator(req)
        if op is None:
            return _err(401, "missing or invalid client credentials", "invalid_api_key")
        try:
            return await fn(await req.json(), op)
        except InsufficientQuota as e:
            return {"rejected": {"kind": "insufficient_quota", "requested": e.requested, "available": e.available}}
        except LedgerError as e:
            return _err(e.status, str(e), e.code)
        except (KeyError, TypeError, ValueError) as e:
            return _err(400, f"bad request: {e}", "invalid_request_error")

    @app.post("/authz/v1/resolve")
    async def resolve(req: Request):
        async def f(b, op):
            p = L.resolve_key(b["api_key"])
            if p is None:
                return _err(401, "unknown or inactive API key", "invalid_api_key")
            return {"principal": {"account_id": p["account_id"], "key_id": p["key_id"]},
                    "snapshot": {"hard_cap": p["hard_cap"], "spent": p["spent"], "reserved": p["reserved"]}}
        return await authz(req, f)

    @app.post("/authz/v1/reserve")
    async def reserve(req: Request):
        async def f(b, op):
            return {"reservation_id": L.reserve(b["account_id"], b["key_id"], int(b["max_tokens"]))}
        return await authz(req, f)

    @app.post("/authz/v1/settle")
    async def settle(req: Request):
        async def f(b, op):
            L.settle(int(b["reservation_id"]), int(b["actual_tokens"]))
            return {"ok": True}
        return await authz(req, f)

    @app.post("/authz/v1/release")
    async def release(req: Request):
        async def f(b, op):
            L.release(int(b["reservation_id"]))
            return {"ok": True}
        return await authz(req, f)

    @app.post("/authz/v1/snapshot")
    async def snapshot(req: Request):
        async def f(b, op):
            return L.snapshot(b["account_id"], b["key_id"])
        return await authz(req, f)

    @app.post("/authz/v1/served-usage")
    async def served(req: Request):
        async def f(b, op):
            for u in b.get("usage", [b]):
                L.record_served(op, u.get("model", ""), int(u.get("prompt_tokens", 0)),
                                int(u.get("completion_tokens", 0)))
            return {"ok": True}
        return await authz(req, f)

    # ---- web surface ----
    def session(req: Request) -> str | None:
        return L.session_account(bearer(req))

    @app.post("/web/v1/register")
    async def register(req: Request):
        b = await req.json()
        email, pw = b.get("email", ""), b.get("password", "")
        if "@" not in email or len(pw) < 8:
            return _err(400, "a valid email and a password of at least 8 characters are required", "invalid_request")
        try:
            aid = L.create_account(email, cfg.signup_allocation, pw)
        except sqlite3.IntegrityError:
            return _err(409, "email already registered", "conflict")
        return {"account_id": aid, "session": L.new_session(aid)}

    @app.post("/web/v1/login")
    async def login(req: Request):
        b = await req.json()
        aid = L.check_password(b.get("email", ""), b.get("password", ""))
        if aid is None:
            return _err(401, "invalid credentials", "invalid_credentials")
        return {"account_id": aid, "session": L.new_session(aid)}

    @app.get("/web/v1/account")
    async def account(req: Request):
        aid = session(req)
        return _err(401, "not signed in", "unauthorized") if aid is None else L.account(aid)

    @app.get("/web/v1/allocation")
    async def allocation(req: Request):
        aid = session(req)
        if aid is None:
            return _err(401, "not signed in", "unauthorized")
        a = L.account(aid)
        return {"total": a["allocation_total"], "spent": a["allocation_spent"], "reserved": a["allocation_reserved"],
                "available": a["allocation_total"] - a["allocation_spent"] - a["allocation_reserved"]}

    @app.get("/web/v1/keys")
    async def keys(req: Request):
        aid = session(req)
        return _err(401, "not signed in", "unauthorized") if aid is None else {"keys": L.list_keys(aid)}

    @app.post("/web/v1/keys")
    async def create_key(req: Request):
        aid = session(req)
        if aid is None:
            return _err(401, "not signed in", "unauthorized")
        b = await req.json()
        try:
            kid, raw = L.create_key(aid, b.get("label", ""), b.get("limit_kind", "percent"),
                                    int(b.get("limit_value", 100)))
        except LedgerError as e:
            return _err(400, str(e), e.code)
        return {"id": kid, "key": raw}

    @app.post("/web/v1/keys/{key_id}/archive")
    async def archive(key_id: str, req: Request):
        aid = session(req)
        if aid is None:
            return _err(401, "not signed in", "unauthorized")
        return {"ok": True} if L.archive_key(aid, key_id) else _err(404, "key not found", "not_found")

    @app.post("/web/v1/redeem")
    async def redeem(req: Request):
        aid = session(req)
        if aid is None:
            return _err(401, "not signed in", "unauthorized")
        try:
            return {"added": L.redeem(aid, (await req.json()).get("code", ""))}
        except LedgerError as e:
            return _err(400, str(e), "invalid_code")

    @app.get("/health")
    async def health():
        return {"status": "ok", "service": "helexa-upstream"}

    return app
