"""Tool-execution service behind the chat app's grounding tools: `GET /fetch?url=` reads
a web page for the model, guarded against server-side request forgery, and returns
its readable text (the reference's crates/helexa-tools: ssrf.rs, fetch.rs, lib.rs).

SSRF rules:
* http / https only, a host is required;
* literal IPs must be globally routable (no loopback, private, link-local, CGNAT
  100.64/10, benchmarking 198.18/15, documentation, multicast, reserved 240/4,
  0/8, 192.0.0/24, IPv6 ULA fc00::/7, link-local fe80::/10, 2001:db8::/32; IPv4-mapped
  IPv6 is judged as its IPv4);
* names must contain a dot and not end in .internal / .local / .lan / .home.arpa;
* every address a name resolves to must pass the IP rule, and the connection goes to
  that validated address (the host header keeps the name), so a second DNS answer
  cannot swap in an internal address; redirects are followed by hand (at most
  `max_redirects`) and every hop is checked again.
Bodies are capped at `max_body_bytes`; text/html (or no content type) is reduced to
readable text, text/plain passes through; anything else is 415. Text is truncated to
`max_text_chars` characters.
"""
from __future__ import annotations

import ipaddress
import re
import socket
from dataclasses import dataclass
from html.parser import HTMLParser
from urllib.parse import urljoin, urlsplit

import httpx
from fastapi import FastAPI
from fastapi.responses import JSONResponse

USER_AGENT = "helexa-b200-tools/0.1 (web_search grounding fetcher)"
BLOCKED_SUFFIXES = (".internal", ".local", ".lan", ".home.arpa")


@dataclass
class ToolsConfig:
    fetch_timeout_s: float = 20.0
    max_body_bytes: int = 2 * 1024 * 1024
    max_text_chars: int = 12_000
    max_redirects: int = 5


class FetchError(Exception):
    status = 502


class Denied(FetchError):
    status = 400


class Unsupported(FetchError):
    status = 415


_V4_DENY = [ipaddress.ip_network(n) for n in (
    "0.0.0.0/8", "10.0.0.0/8", "100.64.0.0/10", "127.0.0.0/8", "169.254.0.0/16", "172.16.0.0/12",
    "192.0.0.0/24", "192.0.2.0/24", "192.168.0.0/16", "198.18.0.0/15", "198.51.100.0/24", "203.0.113.0/24",
    "224.0.0.0/4", "240.0.0.0/4")]
_V6_DENY = [ipaddress.ip_network(n) for n in ("::/128", "::1/128", "fc00::/7", "fe80::/10", "ff00::/8",
                                               "2001:db8::/32")]


def ip_allowed(ip: str | ipaddress._BaseAddress) -> bool:
    a = ipaddress.ip_address(ip) if isinstance(ip, str) else ip
    if a.version == 6 and a.ipv4_mapped is not None:
        a = a.ipv4_mapped
    deny = _V4_DENY if a.version == 4 else _V6_DENY
    return not any(a in n for n in deny)


def check_url(url: str) -> tuple[str, int]:
    """(host, port) of a URL that passes the static rules; raises Denied."""
    parts = urlsplit(url)
    if parts.scheme not in ("http", "https"):
        raise Denied("only http/https URLs are fetchable")
    host = parts.hostname
    if not host:
        raise Denied("URL has no host")
    port = parts.port or (443 if parts.scheme == "https" else 80)
    try:
        a = ipaddress.ip_address(host)
    except ValueError:
        h = host.lower().rstrip(".")
        if "." not in h or any(h.endswith(s) or h == s.lstrip(".") for s in BLOCKED_SUFFIXES):
            raise Denied(f"host '{host}' is not a public hostname") from None
        return host, port
    if not ip_allowed(a):
        raise Denied(f"address {a} is not globally routable")
    return host, port


def resolve_validated(host: str, port: int, resolver=socket.getaddrinfo) -> str:
    """The first resolved address of `host`, after checking that EVERY resolved address
    is allowed (a name with one internal answer is refused outright)."""
    try:
        infos = resolver(host, port, type=socket.SOCK_STREAM)
    except OSError:
        raise Denied(f"host '{host}' did not resolve") from None
    addrs = [i[4][0] for i in infos]
    if not addrs:
        raise Denied(f"host '{host}' did not resolve")
    for a in addrs:
        if not ip_allowed(a):
            raise Denied(f"address {a} is not globally routable")
    return addrs[0]


class _Readable(HTMLParser):
    """Title and block text of a page, without script / style / navigation chrome."""

    SKIP = {"script", "style", "noscript", "nav", "header", "footer", "aside", "form", "svg", "template", "iframe"}
    BLOCK = {"p", "div", "section", "article", "li", "h1", "h2", "h3", "h4", "h5", "h6", "br", "tr", "pre",
             "blockquote", "main"}

    def __init__(self):
        super().__init__(convert_charrefs=True)
        self.title, self.parts, self._skip, self._in_title = "", [], 0, False

    def handle_starttag(self, tag, attrs):
        if tag in self.SKIP:
            self._skip += 1
        elif tag == "title":
            self._in_title = True
        elif tag in self.BLOCK:
            self.parts.append("\n")

    def handle_endtag(self, tag):
        if tag in self.SKIP and self._skip:
            self._skip -= 1
        elif tag == "title":
            self._in_title = False
        elif tag in self.BLOCK:
            self.parts.append("\n")

    def handle_data(self, data):
        if self._in_title:
            self.title += data
        elif not self._skip:
            self.parts.append(data)


def extract_readable(html: str) -> tuple[str, str]:
    p = _Readable()
    p.feed(html)
    p.close()
    text = "".join(p.parts)
    lines = [re.sub(r"[ \t\r\f\v]+", " ", ln).strip() for ln in text.split("\n")]
    text = "\n".join(ln for ln in lines if ln)
    return p.title.strip(), text


def truncate_chars(s: str, n: int) -> tuple[str, bool]:
    return (s, False) if len(s) <= n else (s[:n], True)


async def fetch_page(url: str, cfg: ToolsConfig, client: httpx.AsyncClient | None = None,
                     resolver=socket.getaddrinfo) -> dict:
    own = client is None
    client = client or httpx.AsyncClient(timeout=cfg.fetch_timeout_s, follow_redirects=False)
    try:
        for _ in range(cfg.max_redirects + 1):
            host, port = check_url(url)
            ip = resolve_validated(host, port, resolver)
            parts = urlsplit(url)
            netloc_ip = f"[{ip}]" if ":" in ip else ip
            pinned = parts._replace(netloc=f"{netloc_ip}:{port}").geturl()
            headers = {"Host": parts.netloc.rsplit("@", 1)[-1], "User-Agent": USER_AGENT}
            ext = {"sni_hostname": host} if parts.scheme == "https" else {}
            try:
                async with client.stream("GET", pinned, headers=headers, extensions=ext) as resp:
                    if 300 <= resp.status_code < 400:
                        loc = resp.headers.get("location")
                        if not loc:
                            raise FetchError(f"upstream returned status {resp.status_code}")
                        url = urljoin(url, loc)
                        continue
                    if resp.status_code >= 400:
                        raise FetchError(f"upstream returned status {resp.status_code}")
                    ctype = resp.headers.get("content-type", "").lower()
                    is_html = ctype.startswith("text/html") or ctype.startswith("application/xhtml+xml") or not ctype
                    is_plain = ctype.startswith("text/plain")
                    if not (is_html or is_plain):
                        raise Unsupported(f"unsupported content-type '{ctype}' (text/html or text/plain only)")
                    buf = bytearray()
                    async for chunk in resp.aiter_bytes():
                        buf += chunk[:cfg.max_body_bytes - len(buf)]
                        if len(buf) >= cfg.max_body_bytes:
                            break
            except httpx.HTTPError as e:
                raise FetchError(f"fetch failed: {e}") from None
            body = bytes(buf).decode("utf-8", errors="replace")
            if is_plain:
                text, trunc = truncate_chars(body, cfg.max_text_chars)
                return {"url": url, "title": "", "text": text, "truncated": trunc}
            title, text = extract_readable(body)
            text, trunc = truncate_chars(text, cfg.max_text_chars)
            return {"url": url, "title": title, "text": text, "truncated": trunc}
        raise FetchError("too many redirects")
    finally:
        if own:
            await client.aclose()


def create_tools_app(cfg: ToolsConfig | None = None, transport=None, resolver=socket.getaddrinfo) -> FastAPI:
    cfg = cfg or ToolsConfig()
    app = FastAPI(title="helexa-b200 tools")
    client = httpx.AsyncClient(timeout=cfg.fetch_timeout_s, follow_redirects=False, transport=transport)

    @app.get("/health")
    async def health():
        return {"status": "ok", "service": "helexa-tools"}

    @app.get("/fetch")
    async def fetch(url: str):
        try:
            return await fetch_page(url, cfg, client, resolver)
        except FetchError as e:
            return JSONResponse({"error": str(e)}, status_code=e.status)

    @app.on_event("shutdown")
    async def _stop():
        await client.aclose()

    return app
