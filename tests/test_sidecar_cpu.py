"""The sidecar's request handling without a GPU: health, unknown paths and malformed JSON or
binary bodies are answered before any codec runs (the reference's 400/404 contract,
sidecar.py:119-220), and the binary framing helpers split and rebuild arrays exactly."""

import json
import urllib.error
import urllib.request

import numpy as np
import pytest
import torch

from prismkv_b200 import sidecar


@pytest.fixture(scope="module")
def server():
    srv = sidecar.PrismKVSidecar(port=0)
    srv.start_background()
    yield f"http://127.0.0.1:{srv.port}"
    srv.stop()


def _post(url, body: bytes, headers):
    req = urllib.request.Request(url, data=body, headers=headers, method="POST")
    try:
        with urllib.request.urlopen(req, timeout=30) as r:
            return r.status, r.read(), dict(r.headers)
    except urllib.error.HTTPError as e:
        return e.code, e.read(), dict(e.headers)


def test_health_and_unknown_paths(server):
    with urllib.request.urlopen(server + "/health", timeout=30) as r:
        assert json.loads(r.read()) == {"status": "ok", "version": sidecar.VERSION}
    code, body, _ = _post(server + "/nope", b"{}", {"Content-Type": "application/json"})
    assert code == 404 and "Unknown endpoint" in json.loads(body)["error"]


@pytest.mark.parametrize("path,body,msg", [
    ("/compress", b"", "Empty request body"),
    ("/compress", b"{not json", "JSON parse error"),
    ("/compress", json.dumps({"k": [1.0, 2.0], "v": [1.0, 2.0]}).encode(), "2-D"),
    ("/compress", json.dumps({"v": [[1.0]]}).encode(), "Invalid k/v"),
    ("/decompress", json.dumps({"k_codes": [[1]], "v_codes": [[1]]}).encode(), "Invalid codes or head_dim"),
])
def test_malformed_json_is_refused(server, path, body, msg):
    code, out, _ = _post(server + path, body, {"Content-Type": "application/json"})
    assert code == 400 and msg in json.loads(out)["error"]


@pytest.mark.parametrize("headers,body,msg", [
    ({"X-PrismKV-Shape": "2"}, b"\0" * 16, "X-PrismKV-Shape"),
    ({"X-PrismKV-Shape": "2,64"}, b"\0" * 16, "expected 2 x 2 x 64 x 4"),
    ({"X-PrismKV-Shape": "2,64", "X-PrismKV-Dtype": "int8"}, b"\0" * 1024, "X-PrismKV-Dtype"),
    ({"X-PrismKV-Shape": "2,64", "X-PrismKV-Bits": "4,4"}, b"\0" * 1024, "X-PrismKV-Bits"),
])
def test_malformed_binary_is_refused(server, headers, body, msg):
    code, out, _ = _post(server + "/compress", body, dict(headers, **{"Content-Type": sidecar.BINARY}))
    assert code == 400 and msg in json.loads(out)["error"]


@pytest.mark.parametrize("dtype", ["float32", "float16", "bfloat16"])
def test_binary_framing_round_trips(dtype):
    dt = sidecar.DTYPES[dtype]
    k = torch.randn(5, 64).to(dt)
    v = torch.randn(5, 64).to(dt)
    body = sidecar.tensor_bytes(k) + sidecar.tensor_bytes(v)
    kb, vb = sidecar.split_pair(body, 5, 64, 4 if dt == torch.float32 else 2)
    assert torch.equal(sidecar.floats_from_bytes(kb, 5, 64, dt), k)
    assert torch.equal(sidecar.floats_from_bytes(vb, 5, 64, dt), v)
    assert sidecar.parse_shape("5,64", "s") == (5, 64) and sidecar.parse_bits("3,3,2") == (3, 3, 2)
