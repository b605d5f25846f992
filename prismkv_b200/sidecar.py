"""PrismKVSidecar -- the HTTP compression service, with a binary transport.

Same service as the reference's sidecar (sidecar.py:1-331): ``POST /compress``,
``POST /decompress`` and ``GET /health``, with the same JSON request and response
bodies, so a client written for the reference works unchanged.  The codec behind
it is the GPU backend (``PrismKVBackend``): vectors are encoded and codes decoded
by the kernels, one backend per (head_dim, bits) as in the reference
(sidecar.py:203-211).

The JSON bodies carry every float and code as a decimal list, which costs far more
than the codec itself.  A request whose ``Content-Type`` is
``application/x-prismkv`` carries raw little-endian arrays instead:

* ``POST /compress`` -- body: K then V, each (N, head_dim) row-major;
  headers ``X-PrismKV-Shape: N,head_dim``, ``X-PrismKV-Dtype: float32 |
  float16 | bfloat16`` (default float32), optional ``X-PrismKV-Bits:
  bits_z,bits_r,bits_theta`` (default 4,4,4).  Response body: K codes then V
  codes, each (N, n_groups) int16; headers ``X-PrismKV-Shape: N,n_groups``
  and ``X-PrismKV-Head-Dim``.
* ``POST /decompress`` -- body: K codes then V codes, (N, n_groups) int16
  each; headers ``X-PrismKV-Shape: N,n_groups``, ``X-PrismKV-Head-Dim``
  (the unpadded head_dim), optional ``X-PrismKV-Bits`` and
  ``X-PrismKV-Dtype`` (the output type, default float32).  Response body: K
  then V, (N, head_dim) each.

Malformed requests get the reference's answers: 400 with ``{"error": ...}``
(JSON) for bad bodies, 404 for unknown paths.
"""

from __future__ import annotations

import json
import threading
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
from typing import Any, Dict, Optional, Tuple

import numpy as np
import torch

from .cache.backend import PrismKVBackend
from .cache.cache_config import PrismKVConfig

VERSION = "1.0.0"
BINARY = "application/x-prismkv"
DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}
_ITEM = {torch.float32: 4, torch.float16: 2, torch.bfloat16: 2}


class RequestError(ValueError):
    """A malformed request (answered with 400)."""


def parse_shape(text: Optional[str], what: str) -> Tuple[int, int]:
    try:
        a, b = (int(v) for v in (text or "").split(","))
    except ValueError:
        raise RequestError(f"{what} must be 'rows,cols', got {text!r}") from None
    if a < 0 or b <= 0:
        raise RequestError(f"{what} must be non-negative rows and positive cols, got {text!r}")
    return a, b


def parse_bits(text: Optional[str]) -> Tuple[int, int, int]:
    if not text:
        return 4, 4, 4
    try:
        bz, br, bt = (int(v) for v in text.split(","))
    except ValueError:
        raise RequestError(f"X-PrismKV-Bits must be 'bits_z,bits_r,bits_theta', got {text!r}") from None
    return bz, br, bt


def split_pair(body: bytes, rows: int, cols: int, itemsize: int) -> Tuple[bytes, bytes]:
    """The two equal (rows, cols) arrays of a binary body."""
    one = rows * cols * itemsize
    if len(body) != 2 * one:
        raise RequestError(f"body holds {len(body)} bytes, expected 2 x {rows} x {cols} x {itemsize} = {2 * one}")
    return body[:one], body[one:]


def floats_from_bytes(raw: bytes, rows: int, cols: int, dtype: torch.dtype) -> torch.Tensor:
    if dtype == torch.bfloat16:
        return torch.frombuffer(bytearray(raw), dtype=torch.int16).view(torch.bfloat16).reshape(rows, cols)
    return torch.frombuffer(bytearray(raw), dtype=dtype).reshape(rows, cols) if raw else \
        torch.empty((rows, cols), dtype=dtype)


def tensor_bytes(t: torch.Tensor) -> bytes:
    t = t.contiguous().cpu()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return t.numpy().tobytes()


class _Handler(BaseHTTPRequestHandler):
    backends: Dict[Tuple[int, int, int, int], PrismKVBackend] = {}
    lock = threading.Lock()

    def log_message(self, fmt: str, *args: Any) -> None:      # no access log
        pass

    # -- routing -----------------------------------------------------------
    def do_GET(self) -> None:
        if self.path == "/health":
            self._json(200, {"status": "ok", "version": VERSION})
        else:
            self._json(404, {"error": f"Unknown endpoint: {self.path}"})

    def do_POST(self) -> None:
        if self.path not in ("/compress", "/decompress"):
            self._json(404, {"error": f"Unknown endpoint: {self.path}"})
            return
        length = int(self.headers.get("Content-Length", 0))
        if length == 0:
            self._json(400, {"error": "Empty request body"})
            return
        raw = self.rfile.read(length)
        binary = self.headers.get("Content-Type", "").split(";")[0].strip() == BINARY
        try:
            if binary:
                (self._compress_binary if self.path == "/compress" else self._decompress_binary)(raw)
            else:
                try:
                    body = json.loads(raw)
                except ValueError as e:
                    raise RequestError(f"JSON parse error: {e}") from None
                (self._compress_json if self.path == "/compress" else self._decompress_json)(body)
        except RequestError as e:
            self._json(400, {"error": str(e)})

    # -- endpoints -----------------------------------------------------------
    def _compress_json(self, body: dict) -> None:
        try:
            k = torch.tensor(body["k"], dtype=torch.float32)
            v = torch.tensor(body["v"], dtype=torch.float32)
        except (KeyError, ValueError, TypeError, RuntimeError) as e:
            raise RequestError(f"Invalid k/v: {e}") from None
        if k.dim() != 2 or v.dim() != 2:
            raise RequestError("k and v must be 2-D arrays (N, head_dim)")
        bits = (int(body.get("bits_z", 4)), int(body.get("bits_r", 4)), int(body.get("bits_theta", 4)))
        backend = self._backend(k.shape[1], bits)
        kc, vc = backend.compress(k, v)
        self._json(200, {"k_codes": kc.tolist(), "v_codes": vc.tolist(), "head_dim": k.shape[1],
                         "n_groups": backend.n_groups, "bits_per_dim": sum(bits) / 3})

    def _decompress_json(self, body: dict) -> None:
        try:
            kc = torch.tensor(body["k_codes"], dtype=torch.int16)
            vc = torch.tensor(body["v_codes"], dtype=torch.int16)
            head_dim = int(body["head_dim"])
        except (KeyError, ValueError, TypeError) as e:
            raise RequestError(f"Invalid codes or head_dim: {e}") from None
        if kc.dim() != 2 or vc.dim() != 2:
            raise RequestError("k_codes and v_codes must be 2-D arrays (N, n_groups)")
        bits = (int(body.get("bits_z", 4)), int(body.get("bits_r", 4)), int(body.get("bits_theta", 4)))
        k, v = self._backend(head_dim, bits).decompress(kc, vc)
        self._json(200, {"k": k.tolist(), "v": v.tolist()})

    def _compress_binary(self, raw: bytes) -> None:
        rows, head_dim = parse_shape(self.headers.get("X-PrismKV-Shape"), "X-PrismKV-Shape")
        dtype = DTYPES.get(self.headers.get("X-PrismKV-Dtype", "float32"))
        if dtype is None:
            raise RequestError(f"X-PrismKV-Dtype must be one of {sorted(DTYPES)}")
        bits = parse_bits(self.headers.get("X-PrismKV-Bits"))
        kb, vb = split_pair(raw, rows, head_dim, _ITEM[dtype])
        backend = self._backend(head_dim, bits)
        kc, vc = backend.compress(floats_from_bytes(kb, rows, head_dim, dtype),
                                  floats_from_bytes(vb, rows, head_dim, dtype))
        self._binary(tensor_bytes(kc) + tensor_bytes(vc),
                     {"X-PrismKV-Shape": f"{rows},{backend.n_groups}", "X-PrismKV-Head-Dim": str(head_dim)})

    def _decompress_binary(self, raw: bytes) -> None:
        rows, groups = parse_shape(self.headers.get("X-PrismKV-Shape"), "X-PrismKV-Shape")
        try:
            head_dim = int(self.headers.get("X-PrismKV-Head-Dim", ""))
        except ValueError:
            raise RequestError("X-PrismKV-Head-Dim must be an integer") from None
        dtype = DTYPES.get(self.headers.get("X-PrismKV-Dtype", "float32"))
        if dtype is None:
            raise RequestError(f"X-PrismKV-Dtype must be one of {sorted(DTYPES)}")
        bits = parse_bits(self.headers.get("X-PrismKV-Bits"))
        backend = self._backend(head_dim, bits)
        if groups != backend.n_groups:
            raise RequestError(f"{groups} code groups do not match head_dim {head_dim} ({backend.n_groups})")
        kb, vb = split_pair(raw, rows, groups, 2)
        kc = torch.frombuffer(bytearray(kb), dtype=torch.int16).reshape(rows, groups) if rows else \
            torch.empty((0, groups), dtype=torch.int16)
        vc = torch.frombuffer(bytearray(vb), dtype=torch.int16).reshape(rows, groups) if rows else \
            torch.empty((0, groups), dtype=torch.int16)
        k, v = backend.decompress(kc, vc)
        self._binary(tensor_bytes(k.to(dtype)) + tensor_bytes(v.to(dtype)),
                     {"X-PrismKV-Shape": f"{rows},{head_dim}", "X-PrismKV-Dtype": self.headers.get(
                         "X-PrismKV-Dtype", "float32")})

    # -- helpers -------------------------------------------------------------
    def _backend(self, head_dim: int, bits: Tuple[int, int, int]) -> PrismKVBackend:
        key = (head_dim, *bits)
        with self.lock:
            if key not in self.backends:
                try:
                    cfg = PrismKVConfig(bits_z=bits[0], bits_r=bits[1], bits_theta=bits[2])
                    self.backends[key] = PrismKVBackend(cfg, head_dim=head_dim)
                except (ValueError, AssertionError) as e:
                    raise RequestError(f"Invalid configuration: {e}") from None
            return self.backends[key]

    def _json(self, status: int, payload: dict) -> None:
        body = json.dumps(payload).encode()
        self.send_response(status)
        self.send_header("Content-Type", "application/json")
        self.send_header("Content-Length", str(len(body)))
        self.end_headers()
        self.wfile.write(body)

    def _binary(self, body: bytes, headers: Dict[str, str]) -> None:
        self.send_response(200)
        self.send_header("Content-Type", BINARY)
        self.send_header("Content-Length", str(len(body)))
        for k, v in headers.items():
            self.send_header(k, v)
        self.end_headers()
        self.wfile.write(body)


class PrismKVSidecar:
    """The service (sidecar.py:225-296): ``start()`` blocks; ``start_background()`` serves from a
    thread until ``stop()``.  ``port=0`` binds a free port (``self.port`` then holds it)."""

    def __init__(self, host: str = "127.0.0.1", port: int = 8765) -> None:
        self.host, self.port = host, port
        self._server: Optional[ThreadingHTTPServer] = None
        self._thread: Optional[threading.Thread] = None

    def _bind(self) -> ThreadingHTTPServer:
        srv = ThreadingHTTPServer((self.host, self.port), _Handler)
        self.port = srv.server_address[1]
        return srv

    def start(self) -> None:
        self._server = self._bind()
        print(f"PrismKV sidecar running at http://{self.host}:{self.port}")
        try:
            self._server.serve_forever()
        except KeyboardInterrupt:
            pass
        finally:
            self._server.server_close()

    def start_background(self) -> None:
        self._server = self._bind()
        self._thread = threading.Thread(target=self._server.serve_forever, daemon=True)
        self._thread.start()

    def stop(self) -> None:
        if self._server is not None:
            self._server.shutdown()
            self._server.server_close()
            self._server = None


def _main() -> None:
    import argparse
    ap = argparse.ArgumentParser(description="PrismKV sidecar: HTTP KV compression on the GPU")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8765)
    args = ap.parse_args()
    PrismKVSidecar(host=args.host, port=args.port).start()


if __name__ == "__main__":
    _main()


__all__ = ["PrismKVSidecar", "BINARY", "VERSION"]
