"""Confidential document portal (the reference's crates/helexa-angels): investors sign in
with their platform account and read the documents of funding rounds they were
invited to.

The design follows from one requirement, knowing which named person read which
version of which document:
* pages are rendered on the server, so an unauthenticated request can only obtain the
  sign-in form, and one document view is one request (the audit log records reading,
  not fetching);
* access attaches to a user through a grant (pending / active / revoked), never to a
  URL; an invite code only lets its holder identify themselves (a forwarded code yields
  another named account, not anonymous access), and unknown, revoked, expired and used
  up codes are indistinguishable to the visitor;
* every document page carries the viewer's identity and the time as a watermark, and
  every view is logged with the document's content version (a hash of its body); the
  log keeps the email beside the user id so it outlives the account;
* credentials are the platform's (the account ledger's password check), sessions are
  the portal's own cookies, so a platform session never opens the portal.

Administration (rounds, documents, invites, approving grants) is a Python API, not a
web surface.
"""
from __future__ import annotations

import hashlib
import html
import secrets
import sqlite3
import threading
import time

from fastapi import FastAPI, Request
from fastapi.responses import HTMLResponse, RedirectResponse

from .upstream import Ledger, sha256

SCHEMA = """
CREATE TABLE IF NOT EXISTS rounds (slug TEXT PRIMARY KEY, title TEXT, status TEXT NOT NULL DEFAULT 'open');
CREATE TABLE IF NOT EXISTS documents (round TEXT, slug TEXT, title TEXT, body TEXT, version TEXT,
  PRIMARY KEY (round, slug));
CREATE TABLE IF NOT EXISTS invites (code_hash BLOB PRIMARY KEY, round TEXT, label TEXT, auto_grant INTEGER,
  uses_left INTEGER, expires REAL, revoked INTEGER NOT NULL DEFAULT 0);
CREATE TABLE IF NOT EXISTS grants (account_id TEXT, round TEXT, state TEXT, granted_at REAL, via TEXT,
  PRIMARY KEY (account_id, round));
CREATE TABLE IF NOT EXISTS audit (id INTEGER PRIMARY KEY AUTOINCREMENT, ts REAL, account_id TEXT, email TEXT,
  round TEXT, document TEXT, version TEXT, kind TEXT, ip TEXT, user_agent TEXT);
CREATE TABLE IF NOT EXISTS portal_sessions (token_hash BLOB PRIMARY KEY, account_id TEXT, expires REAL);
"""
COOKIE = "portal_session"
INVITE_COOKIE = "portal_invite"


class Portal:
    def __init__(self, ledger: Ledger, path: str = ":memory:", session_ttl_s: float = 8 * 3600):
        self.ledger = ledger
        self.db = sqlite3.connect(path, check_same_thread=False, isolation_level=None)
        self.db.row_factory = sqlite3.Row
        self.db.executescript(SCHEMA)
        self.ttl = session_ttl_s
        self._lock = threading.Lock()

    def _exec(self, sql: str, args=()):
        with self._lock:
            return self.db.execute(sql, args)

    # ---- administration ----
    def create_round(self, slug: str, title: str):
        self._exec("INSERT OR REPLACE INTO rounds (slug, title, status) VALUES (?, ?, 'open')", (slug, title))

    def put_document(self, round_slug: str, slug: str, title: str, body: str) -> str:
        version = hashlib.sha256(body.encode()).hexdigest()[:16]
        self._exec("INSERT OR REPLACE INTO documents VALUES (?, ?, ?, ?, ?)", (round_slug, slug, title, body, version))
        return version

    def mint_invite(self, round_slug: str, label: str = "", auto_grant: bool = False, uses: int = 50,
                    ttl_s: float = 30 * 86400) -> str:
        code = secrets.token_urlsafe(12)
        self._exec("INSERT INTO invites VALUES (?, ?, ?, ?, ?, ?, 0)",
                   (sha256(code), round_slug, label, int(auto_grant), uses, time.time() + ttl_s))
        return code

    def revoke_invite(self, code: str):
        self._exec("UPDATE invites SET revoked = 1 WHERE code_hash = ?", (sha256(code),))

    def set_grant(self, account_id: str, round_slug: str, state: str, via: str = "admin"):
        if state not in ("pending", "active", "revoked"):
            raise ValueError(state)
        self._exec("INSERT INTO grants VALUES (?, ?, ?, ?, ?) ON CONFLICT(account_id, round) DO UPDATE SET "
                   "state = excluded.state, granted_at = excluded.granted_at", (account_id, round_slug, state,
                                                                              time.time(), via))

    def audit_log(self) -> list[dict]:
        return [dict(r) for r in self._exec("SELECT * FROM audit ORDER BY id")]

    # ---- visitor side ----
    def redeem_invite(self, account_id: str, code: str) -> str | None:
        """Grant (active or pending) from a live code, or None; a dead code and an unknown
        one look the same to the caller."""
        with self._lock:
            r = self.db.execute("SELECT round, auto_grant, uses_left, expires, revoked FROM invites WHERE code_hash = ?",
                                (sha256(code),)).fetchone()
            if r is None or r["revoked"] or r["uses_left"] <= 0 or r["expires"] < time.time():
                return None
            self.db.execute("UPDATE invites SET uses_left = uses_left - 1 WHERE code_hash = ?", (sha256(code),))
            cur = self.db.execute("SELECT state FROM grants WHERE account_id = ? AND round = ?",
                                  (account_id, r["round"])).fetchone()
        if cur is None or cur["state"] == "pending":
            self.set_grant(account_id, r["round"], "active" if r["auto_grant"] else "pending", via="invite")
        return r["round"]

    def grant_state(self, account_id: str, round_slug: str) -> str | None:
        r = self._exec("SELECT state FROM grants WHERE account_id = ? AND round = ?", (account_id, round_slug)).fetchone()
        return r["state"] if r else None

    def rounds_for(self, account_id: str) -> list[dict]:
        return [dict(r) for r in self._exec(
            "SELECT r.slug, r.title, g.state FROM grants g JOIN rounds r ON r.slug = g.round "
            "WHERE g.account_id = ? AND g.state != 'revoked' ORDER BY r.slug", (account_id,))]

    def new_session(self, account_id: str) -> str:
        tok = secrets.token_urlsafe(32)
        self._exec("INSERT INTO portal_sessions VALUES (?, ?, ?)", (sha256(tok), account_id, time.time() + self.ttl))
        return tok

    def session_account(self, tok: str | None) -> str | None:
        if not tok:
            return None
        r = self._exec("SELECT account_id, expires FROM portal_sessions WHERE token_hash = ?", (sha256(tok),)).fetchone()
        return r["account_id"] if r and r["expires"] > time.time() else None

    def end_session(self, tok: str | None):
        if tok:
            self._exec("DELETE FROM portal_sessions WHERE token_hash = ?", (sha256(tok),))

    def record(self, request: Request, account_id: str | None, kind: str, round_slug=None, doc=None, version=None):
        email = self.ledger.account(account_id)["email"] if account_id else None
        self._exec("INSERT INTO audit (ts, account_id, email, round, document, version, kind, ip, user_agent) "
                   "VALUES (?, ?, ?, ?, ?, ?, ?, ?, ?)",
                   (time.time(), account_id, email, round_slug, doc, version, kind,
                    request.client.host if request.client else None, request.headers.get("user-agent")))


def _page(title: str, body: str, watermark: str | None = None) -> HTMLResponse:
    wm = ""
    if watermark:
        mark = html.escape(watermark)
        wm = ("<div style='position:fixed;inset:0;pointer-events:none;opacity:.08;font-size:2rem;"
              "transform:rotate(-30deg);display:flex;align-items:center;justify-content:center'>"
              f"{mark}</div><footer class='wm'>Confidential. Viewed by {mark}.</footer>")
    return HTMLResponse(f"<!doctype html><html><head><meta charset='utf-8'><title>{html.escape(title)}</title>"
                        "<meta name='robots' content='noindex'></head><body style='font-family:system-ui;"
                        f"max-width:46rem;margin:2rem auto'>{body}{wm}</body></html>",
                        headers={"Cache-Control": "no-store"})


def create_portal(portal: Portal) -> FastAPI:
    app = FastAPI(title="helexa-b200 document portal")
    app.state.portal = portal
    L = portal.ledger

    def who(request: Request) -> str | None:
        return portal.session_account(request.cookies.get(COOKIE))

    def signin_form(msg: str = "", register: bool = False) -> HTMLResponse:
        action = "/register" if register else "/signin"
        return _page("Sign in", f"<h1>{'Create account' if register else 'Sign in'}</h1>"
                     f"<p>{html.escape(msg)}</p><form method='post' action='{action}'>"
                     "<input name='email' type='email' placeholder='email'> "
                     "<input name='password' type='password' placeholder='password'> <button>go</button></form>"
                     + ("" if register else "<p><a href='/register'>create an account</a></p>"))

    async def after_signin(request: Request, aid: str):
        resp = RedirectResponse("/", status_code=303)
        resp.set_cookie(COOKIE, portal.new_session(aid), httponly=True, samesite="strict", secure=False)
        code = request.cookies.get(INVITE_COOKIE)
        if code:
            portal.redeem_invite(aid, code)
            resp.delete_cookie(INVITE_COOKIE)
        portal.record(request, aid, "signin")
        return resp

    @app.get("/")
    async def home(request: Request):
        aid = who(request)
        if aid is None:
            return signin_form()
        rows = portal.rounds_for(aid)
        items = "".join(f"<li><a href='/r/{html.escape(r['slug'])}'>{html.escape(r['title'])}</a></li>"
                        if r["state"] == "active" else f"<li>{html.escape(r['title'])}: awaiting approval</li>"
                        for r in rows)
        return _page("Portal", f"<h1>Rounds</h1><ul>{items or '<li>No rounds yet.</li>'}</ul>"
                     "<p><a href='/signout'>sign out</a></p>")

    @app.get("/signin")
    async def signin_page():
        return signin_form()

    @app.post("/signin")
    async def signin(request: Request):
        form = await request.form()
        aid = L.check_password(str(form.get("email", "")), str(form.get("password", "")))
        if aid is None:
            return signin_form("Those credentials did not match an account.")
        return await after_signin(request, aid)

    @app.get("/register")
    async def register_page():
        return signin_form(register=True)

    @app.post("/register")
    async def register(request: Request):
        form = await request.form()
        email, pw = str(form.get("email", "")), str(form.get("password", ""))
        if "@" not in email or len(pw) < 8:
            return signin_form("A valid email and a password of at least 8 characters are required.", register=True)
        try:
            aid = L.create_account(email, 0, pw)
        except sqlite3.IntegrityError:
            return signin_form("That email already has an account; sign in instead.")
        return await after_signin(request, aid)

    @app.get("/signout")
    async def signout(request: Request):
        portal.end_session(request.cookies.get(COOKIE))
        resp = RedirectResponse("/", status_code=303)
        resp.delete_cookie(COOKIE)
        return resp

    @app.get("/i/{code}")
    async def enter(code: str, request: Request):
        aid = who(request)
        if aid is None:  # identify first; the code is applied after sign-in
            resp = RedirectResponse("/register", status_code=303)
            resp.set_cookie(INVITE_COOKIE, code, httponly=True, samesite="lax", max_age=3600)
            return resp
        portal.redeem_invite(aid, code)
        return RedirectResponse("/", status_code=303)

    def round_access(request: Request, slug: str):
        aid = who(request)
        if aid is None:
            return None, signin_form()
        if portal.grant_state(aid, slug) != "active":
            portal.record(request, aid, "denied", slug)
            return None, _page("Not available", "<p>This round is not available to your account.</p>")
        return aid, None

    @app.get("/r/{slug}")
    async def round_index(slug: str, request: Request):
        aid, deny = round_access(request, slug)
        if deny is not None:
            return deny
        docs = portal._exec("SELECT slug, title FROM documents WHERE round = ? ORDER BY slug", (slug,)).fetchall()
        items = "".join(f"<li><a href='/r/{html.escape(slug)}/{html.escape(d['slug'])}'>{html.escape(d['title'])}</a>"
                        "</li>" for d in docs)
        portal.record(request, aid, "index", slug)
        return _page(slug, f"<h1>{html.escape(slug)}</h1><ul>{items}</ul>",
                     watermark=f"{L.account(aid)['email']} {time.strftime('%Y-%m-%d %H:%M UTC', time.gmtime())}")

    @app.get("/r/{slug}/{doc}")
    async def document(slug: str, doc: str, request: Request):
        aid, deny = round_access(request, slug)
        if deny is not None:
            return deny
        d = portal._exec("SELECT title, body, version FROM documents WHERE round = ? AND slug = ?", (slug, doc)).fetchone()
        if d is None:
            return _page("Not found", "<p>No such document.</p>")
        portal.record(request, aid, "view", slug, doc, d["version"])
        body = "".join(f"<p>{html.escape(p)}</p>" for p in d["body"].split("\n\n"))
        return _page(d["title"], f"<h1>{html.escape(d['title'])}</h1>{body}"
                     f"<p class='ver'>version {d['version']}</p>",
                     watermark=f"{L.account(aid)['email']} {time.strftime('%Y-%m-%d %H:%M UTC', time.gmtime())}")

    @app.get("/health")
    async def health():
        return {"status": "ok", "service": "helexa-portal"}

    return app
