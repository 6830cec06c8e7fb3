"""The drop-in surface end to end: the reference's own pa::server (phone-attn/phone-attn.h, unmodified) with
pa::cuda_engine as its GPU engine (oracle/_ref/pa-serve-cuda), driven over loopback TCP by the reference's own
`pa-tool test` client, which checks layer 0 against its fp64 reference and prints PASS/FAIL at its 5e-3 gate
(phone-attn/pa-tool.cpp:150-173), plus its ATTN_BIG-vs-ATTN consistency check (phone-attn/pa-tool.cpp:230-238).
Both binaries are built from the reference sources by oracle/Makefile."""
import os
import socket
import subprocess
import time

import pytest

pytestmark = pytest.mark.gpu

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref")
SERVE, TOOL = os.path.join(REF, "pa-serve-cuda"), os.path.join(REF, "pa-tool")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


# pa-tool test's trailing arguments: SME workers, pack helpers, GPU share (permille), GPU chunk, f16 storage
# (phone-attn/pa-tool.cpp:107-112); F16 asks the server to keep the q8_0 rows it receives as f16 pages (store_f16)
F16 = ["1", "1", "0", "1024", "1"]


@pytest.mark.skipif(not (os.path.exists(SERVE) and os.path.exists(TOOL)),
                    reason="oracle/_ref binaries not built (they need the reference tree at build time)")
@pytest.mark.parametrize("env,nkeys,extra", [({}, 16384, []), ({"PA_Q4": "1"}, 16384, []), ({"PA_NTOK": "1"}, 16384, []),
                                             ({"PA_NTOK": "3"}, 8192, []), ({"PA_BIG_TOK": "64"}, 8192, []),
                                             ({"PA_Q4": "1", "PA_BIG_TOK": "24"}, 4096, []), ({}, 8192, F16),
                                             ({"PA_NTOK": "1", "PA_BIG_TOK": "24"}, 4096, F16)])
def test_reference_pa_tool_against_cuda_engine(env, nkeys, extra):
    port = _free_port()
    srv = subprocess.Popen([SERVE, str(port), "2"], stdout=subprocess.DEVNULL, stderr=subprocess.PIPE, text=True)
    try:
        # the server initialises CUDA before it listens: wait until the port accepts a connection
        deadline = time.time() + 60
        while True:
            assert srv.poll() is None, srv.stderr.read()
            try:
                with socket.create_connection(("127.0.0.1", port), timeout=1.0):
                    break
            except OSError:
                if time.time() > deadline:
                    raise
                time.sleep(0.2)
        out = subprocess.run([TOOL, "test", "127.0.0.1", str(port), str(nkeys), "4", "4", *extra], env=dict(os.environ, **env),
                             capture_output=True, text=True, timeout=300)
        text = out.stdout + out.stderr
        assert out.returncode == 0, text
        assert "-> PASS" in text and "FAIL" not in text, text
        assert "engine=pa-cuda" in text, text
        print(text)
    finally:
        srv.kill()
        srv.wait()


CLIENT = os.path.join(REF, "pa-client-check")


@pytest.mark.skipif(not (os.path.exists(SERVE) and os.path.exists(CLIENT)),
                    reason="oracle/_ref binaries not built (they need the reference tree at build time)")
@pytest.mark.parametrize("quant", ["1", "2"])
def test_store_protocol_truncate_fetch_against_cuda_engine(quant):
    """The rest of the store protocol through pa::cuda_engine's managed pages: the reference's own pa::client
    (oracle/_ref/pa-client-check) APPENDs, ATTNs, TRUNCATEs into the middle of a page and to a page boundary, ATTNs over
    the kept keys, FETCHes rows the GPU has read, APPENDs new rows over the truncated range (the cut page rewritten at
    the key count it had before) and ATTNs again; every reply is checked against the fp64 oracle over exactly the keys
    held at that point (pa-tool's 5e-3 gate), every FETCH byte for byte (phone-attn/phone-attn.h:399-465, :766-770)."""
    port = _free_port()
    srv = subprocess.Popen([SERVE, str(port), "2"], stdout=subprocess.DEVNULL, stderr=subprocess.PIPE, text=True)
    try:
        deadline = time.time() + 60
        while True:
            assert srv.poll() is None, srv.stderr.read()
            try:
                with socket.create_connection(("127.0.0.1", port), timeout=1.0):
                    break
            except OSError:
                if time.time() > deadline:
                    raise
                time.sleep(0.2)
        out = subprocess.run([CLIENT, "127.0.0.1", str(port), quant], capture_output=True, text=True, timeout=300)
        text = out.stdout + out.stderr
        print(text)
        assert out.returncode == 0, text
        assert "ALL PASS" in text and "FAIL" not in text, text
        assert "engine=pa-cuda" in text, text
    finally:
        srv.kill()
        srv.wait()
