"""S3-compatible object store for the G4 tier.

``S3ObjectStore`` speaks the S3 REST API directly (``requests`` over a
pooled HTTP session per I/O thread) and signs every request with AWS
Signature Version 4 (HMAC-SHA256 over the canonical request, the scheme
AWS publishes for S3 header authentication), so it works against AWS S3
and S3-compatible services (MinIO, Ceph RGW) with no SDK. It implements the
same ``ObjectBlockOps`` surface as the filesystem store: ``has`` (HEAD),
``put`` (PUT), ``get`` (GET, None on 404), block upload/download between
the pinned G2 pool and objects, and a lock per block for single-writer
uploads.

The lock is an object ``<key>.lock`` holding JSON ``{instance_id,
acquired_at, deadline}``, created with a conditional PUT
(``If-None-Match: *``, so exactly one writer wins); a lock past its deadline
(or unreadable) is taken over with a compare-and-swap PUT
(``If-Match: <etag>`` of the lock that was read), and a lock this instance
already holds counts as acquired.

Parity: crates/kvbm-engine/src/object/s3/client.rs:25-660 (S3Config aws /
minio / path style / concurrency, put_if_not_exists, get_object,
delete_object, has_object, put_object, get_object_with_etag,
put_object_if_match, ensure_bucket_exists, block put/get through the
layout) and s3/lock.rs (S3LockManager: lock and meta keys, deadline,
CAS takeover of expired or malformed locks).
"""

from __future__ import annotations

import ctypes
import datetime as _dt
import hashlib
import hmac
import json
import os
import threading
import uuid
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field
from urllib.parse import quote

from .store import ObjectBlockOps

EMPTY_SHA256 = hashlib.sha256(b"").hexdigest()


@dataclass
class S3Config:
    endpoint_url: str | None = "http://localhost:9000"
    bucket: str = "kvbm-blocks"
    region: str = "us-east-1"
    force_path_style: bool = True
    max_concurrent_requests: int = 16
    access_key: str | None = None
    secret_key: str | None = None
    session_token: str | None = None
    timeout_s: float = 30.0
    extra: dict = field(default_factory=dict)

    @classmethod
    def aws(cls, bucket: str, region: str) -> "S3Config":
        return cls(endpoint_url=None, bucket=bucket, region=region, force_path_style=False)

    @classmethod
    def minio(cls, endpoint_url: str, bucket: str) -> "S3Config":
        return cls(endpoint_url=endpoint_url, bucket=bucket, region="us-east-1", force_path_style=True)

    def credentials(self) -> tuple[str, str, str | None]:
        ak = self.access_key or os.environ.get("AWS_ACCESS_KEY_ID")
        sk = self.secret_key or os.environ.get("AWS_SECRET_ACCESS_KEY")
        tok = self.session_token or os.environ.get("AWS_SESSION_TOKEN")
        if not ak or not sk:
            raise RuntimeError("S3 credentials missing (access_key/secret_key or AWS_ACCESS_KEY_ID/"
                               "AWS_SECRET_ACCESS_KEY)")
        return ak, sk, tok


# ------------------------------------------------------------------ SigV4
def _hmac(key: bytes, msg: str) -> bytes:
    return hmac.new(key, msg.encode(), hashlib.sha256).digest()


def signing_key(secret: str, date: str, region: str, service: str = "s3") -> bytes:
    k = _hmac(("AWS4" + secret).encode(), date)
    k = _hmac(k, region)
    k = _hmac(k, service)
    return _hmac(k, "aws4_request")


def sign_v4(method: str, path: str, query: dict[str, str], headers: dict[str, str], payload_sha256: str,
            access_key: str, secret_key: str, region: str, amz_date: str, service: str = "s3") -> str:
    """The ``Authorization`` header value for a request. ``headers`` must already hold ``host``,
    ``x-amz-date`` and ``x-amz-content-sha256``; every header given is signed."""
    canon_path = quote(path, safe="/~")
    canon_query = "&".join(f"{quote(k, safe='~')}={quote(str(v), safe='~')}" for k, v in sorted(query.items()))
    hs = {k.lower().strip(): " ".join(str(v).split()) for k, v in headers.items()}
    signed = ";".join(sorted(hs))
    canon_headers = "".join(f"{k}:{hs[k]}\n" for k in sorted(hs))
    canonical = "\n".join([method, canon_path, canon_query, canon_headers, signed, payload_sha256])
    date = amz_date[:8]
    scope = f"{date}/{region}/{service}/aws4_request"
    to_sign = "\n".join(["AWS4-HMAC-SHA256", amz_date, scope, hashlib.sha256(canonical.encode()).hexdigest()])
    sig = hmac.new(signing_key(secret_key, date, region, service), to_sign.encode(), hashlib.sha256).hexdigest()
    return f"AWS4-HMAC-SHA256 Credential={access_key}/{scope}, SignedHeaders={signed}, Signature={sig}"


class S3Error(RuntimeError):
    def __init__(self, status: int, method: str, key: str, body: bytes = b""):
        super().__init__(f"S3 {method} {key!r} failed: HTTP {status} {body[:200]!r}")
        self.status = status


class S3ObjectStore(ObjectBlockOps):
    def __init__(self, config: S3Config, instance_id: str | None = None, lock_timeout_s: float = 300.0):
        import requests  # noqa: F401  (fail at construction when the client library is missing)

        self.cfg = config
        self.instance_id = instance_id or uuid.uuid4().hex
        self.lock_timeout_s = lock_timeout_s
        self._creds = config.credentials()
        self._tls = threading.local()
        self._pool = ThreadPoolExecutor(max_workers=max(1, config.max_concurrent_requests),
                                        thread_name_prefix="kvbm-s3")
        self._lock = threading.Lock()
        self.stats = {"puts": 0, "gets": 0, "hits": 0, "misses": 0, "bytes_out": 0, "bytes_in": 0}

    # ------------------------------------------------------------ transport
    def _session(self):
        s = getattr(self._tls, "s", None)
        if s is None:
            import requests

            s = self._tls.s = requests.Session()
        return s

    def _url_parts(self, key: str | None) -> tuple[str, str, str]:
        """(base URL, host header, path) for the bucket or an object in it."""
        if self.cfg.endpoint_url:
            base = self.cfg.endpoint_url.rstrip("/")
        else:
            base = f"https://s3.{self.cfg.region}.amazonaws.com"
        scheme, rest = base.split("://", 1)
        host = rest.split("/", 1)[0]
        obj = "" if key is None else "/" + key
        if self.cfg.force_path_style:
            return f"{scheme}://{host}", host, f"/{self.cfg.bucket}{obj}" if obj else f"/{self.cfg.bucket}"
        vhost = f"{self.cfg.bucket}.{host}"
        return f"{scheme}://{vhost}", vhost, obj or "/"

    def _request(self, method: str, key: str | None, data: bytes | memoryview | None = None,
                 headers: dict | None = None, query: dict | None = None):
        base, host, path = self._url_parts(key)
        body = bytes(data) if data is not None else b""
        sha = hashlib.sha256(body).hexdigest() if body else EMPTY_SHA256
        amz_date = _dt.datetime.now(_dt.timezone.utc).strftime("%Y%m%dT%H%M%SZ")
        ak, sk, tok = self._creds
        h = {"host": host, "x-amz-date": amz_date, "x-amz-content-sha256": sha}
        if tok:
            h["x-amz-security-token"] = tok
        for k, v in (headers or {}).items():
            h[k.lower()] = v
        h["authorization"] = sign_v4(method, path, query or {}, h, sha, ak, sk, self.cfg.region, amz_date)
        url = base + quote(path, safe="/~")
        return self._session().request(method, url, data=body if body else None, params=query or None,
                                       headers=h, timeout=self.cfg.timeout_s)

    # --------------------------------------------------------- bucket / raw
    def ensure_bucket(self) -> None:
        r = self._request("HEAD", None)
        if r.status_code == 200:
            return
        if r.status_code != 404:
            raise S3Error(r.status_code, "HEAD", self.cfg.bucket, r.content)
        r = self._request("PUT", None)
        if r.status_code not in (200, 409):  # 409: created concurrently by someone else
            raise S3Error(r.status_code, "PUT", self.cfg.bucket, r.content)

    def has(self, key: str) -> bool:
        r = self._request("HEAD", key)
        if r.status_code in (200, 404):
            return r.status_code == 200
        raise S3Error(r.status_code, "HEAD", key, r.content)

    def put(self, key: str, data) -> None:
        r = self._request("PUT", key, data)
        if r.status_code != 200:
            raise S3Error(r.status_code, "PUT", key, r.content)
        with self._lock:
            self.stats["puts"] += 1
            self.stats["bytes_out"] += len(data)

    def put_if_not_exists(self, key: str, data) -> bool:
        """Create ``key`` only if absent: True when this call created it, False when it existed."""
        r = self._request("PUT", key, data, headers={"if-none-match": "*"})
        if r.status_code == 200:
            return True
        if r.status_code in (412, 409):
            return False
        raise S3Error(r.status_code, "PUT", key, r.content)

    def put_if_match(self, key: str, data, etag: str) -> bool:
        r = self._request("PUT", key, data, headers={"if-match": etag})
        if r.status_code == 200:
            return True
        if r.status_code in (412, 404):
            return False
        raise S3Error(r.status_code, "PUT", key, r.content)

    def get_with_etag(self, key: str) -> tuple[bytes, str | None] | None:
        r = self._request("GET", key)
        if r.status_code == 404:
            return None
        if r.status_code != 200:
            raise S3Error(r.status_code, "GET", key, r.content)
        return r.content, r.headers.get("ETag")

    def get(self, key: str) -> bytes | None:
        got = self.get_with_etag(key)
        with self._lock:
            self.stats["gets"] += 1
            if got is None:
                self.stats["misses"] += 1
            else:
                self.stats["hits"] += 1
                self.stats["bytes_in"] += len(got[0])
        return None if got is None else got[0]

    def delete(self, key: str) -> bool:
        r = self._request("DELETE", key)
        if r.status_code in (200, 204):
            return True
        if r.status_code == 404:
            return False
        raise S3Error(r.status_code, "DELETE", key, r.content)

    # ----------------------------------------------------------------- locks
    def _lock_body(self) -> bytes:
        now = _dt.datetime.now(_dt.timezone.utc)
        return json.dumps({"instance_id": self.instance_id, "acquired_at": now.isoformat(),
                           "deadline": (now + _dt.timedelta(seconds=self.lock_timeout_s)).isoformat()}).encode()

    def try_lock(self, key: str, ttl_s: float | None = None) -> bool:
        if ttl_s is not None:
            self.lock_timeout_s = ttl_s
        lk = key + ".lock"
        body = self._lock_body()
        if self.put_if_not_exists(lk, body):
            return True
        got = self.get_with_etag(lk)
        if got is None:  # released between the two calls: try once more
            return self.put_if_not_exists(lk, body)
        data, etag = got
        try:
            held = json.loads(data)
            if held["instance_id"] == self.instance_id:
                return True
            expired = _dt.datetime.now(_dt.timezone.utc) > _dt.datetime.fromisoformat(held["deadline"])
        except (ValueError, KeyError, TypeError):
            expired = True  # malformed lock: take it over
        if not expired:
            return False
        if etag:
            return self.put_if_match(lk, body, etag)
        self.put(lk, body)
        return True

    def unlock(self, key: str) -> None:
        self.delete(key + ".lock")

    def has_meta(self, key: str) -> bool:
        return self.has(key + ".meta")

    def put_meta(self, key: str) -> None:
        self.put(key + ".meta", b"")

    # ------------------------------------------------- block <-> pinned G2
    def put_blocks(self, keys: list[str], host_ptrs: list[int], nbytes: int) -> list:
        """Upload pinned-host block regions (returns futures); each upload releases its lock."""
        def one(k, p):
            self.put(k, (ctypes.c_uint8 * nbytes).from_address(p))
            self.unlock(k)
        return [self._pool.submit(one, k, p) for k, p in zip(keys, host_ptrs)]

    def get_blocks(self, keys: list[str], host_ptrs: list[int], nbytes: int) -> list[bool]:
        def one(k, p):
            data = self.get(k)
            if data is None or len(data) != nbytes:
                return False
            ctypes.memmove(p, data, nbytes)
            return True
        return [f.result() for f in [self._pool.submit(one, k, p) for k, p in zip(keys, host_ptrs)]]

    def close(self) -> None:
        self._pool.shutdown(wait=True)
