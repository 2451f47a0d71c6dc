"""Host-side harness: the ``libgpu_scheduler.so`` C API, the benchmark
workloads, and the HP/BE client loop.

It mirrors what the reference's Python drivers do (python/test_orion_blocking.py
``load_library`` 143-189 and ``run_test`` 192-423; python/launch_jobs.py
``OrionScheduler`` 32-127): load the preloaded scheduler library through
ctypes, build the models, warm them up with capture off, register one thread
per client (client 0 = HP, 1.. = BE), start the workers, turn capture on and
run the client loops.  Differences: HP latency is measured per iteration with
CUDA events recorded in the client's stream order (the interposer keeps
``cudaEventRecord`` in order), and BE throughput is measured over the same
window.

Workloads follow the configurations the reference is benchmarked on:
* ``make_gpt``   — the reference's CharGPT (python/GPT.py:27-149): per-head
  q/k/v projections, 6 layers, d_model 512, 8 heads, FFN 2048 with GELU,
  pre-LayerNorm, learned positions, dropout 0.4, vocab 32000.
* ``make_vgg16`` — torchvision VGG16 (13 conv3x3 + ReLU, 5 max-pools,
  FC 25088-4096-4096-1000), Kaiming-normal init.
* ``make_llama`` — the reference's CharLLaMA (python/LLaMA.py): RMSNorm,
  complex rotary embedding, SwiGLU; 12 layers, d_model 2048, 16 heads,
  FFN 5504, vocab 32000.
"""
from __future__ import annotations

import ctypes
import math
import os
import threading
import time

from . import LIBSHIM

# ---------------------------------------------------------------- library ---


class Orion:
    """ctypes view of the scheduler library (the reference driver's API set)."""

    def __init__(self, path: str = LIBSHIM):
        self.lib = ctypes.CDLL(path, mode=ctypes.RTLD_GLOBAL)
        L = self.lib
        I, P = ctypes.c_int, ctypes.c_void_p
        sig = {
            "orion_init_scheduler": ([I], I), "orion_start_scheduler_thread": ([], I),
            "orion_start_scheduler": ([I], I), "orion_stop_scheduler": ([], None),
            "orion_set_client_idx": ([I], None), "orion_get_client_idx": ([], I),
            "orion_load_kernel_info": ([I, ctypes.c_char_p], I),
            "orion_set_client_kernels": ([I, I], None), "orion_set_sm_threshold": ([I], None),
            "orion_get_sm_threshold": ([], I), "orion_sync_client_stream": ([I], None),
            "orion_reset_state": ([], None), "orion_autotune_green_ctx": ([], I),
            "orion_set_capture": ([I], I), "orion_set_enabled": ([I], None),
            "orion_is_enabled": ([], I), "orion_register_client_stream": ([I, P], None),
            "orion_register_client_handle": ([I, P], None),
            "orion_resolve_client_idx": ([P, P], I), "orion_set_async_mode": ([I], None),
            "orion_get_async_mode": ([], I), "orion_init": ([I], I), "orion_shutdown": ([], None),
            "orion_set_be_keep_sms": ([I], None), "orion_get_be_keep_sms": ([], I),
            "orion_set_profile_launches": ([I], None),
            "orion_set_sm_budgets": ([I, I], I),
            "orion_get_client_stats": ([I, ctypes.POINTER(ctypes.c_ulonglong)], I),
            "orion_set_be_host_hold_us": ([I], None), "orion_get_be_host_hold_us": ([], I),
            "orion_get_client_host_holds": ([I], ctypes.c_ulonglong),
            "orion_set_profile_every": ([I], None),
            "orion_load_profile": ([ctypes.c_char_p], I),
            "orion_start_profiling": ([ctypes.c_char_p], None),
            "orion_end_profiling": ([ctypes.c_char_p], None),
            "orion_op_log_start": ([], None), "orion_op_log_end": ([ctypes.c_char_p], I),
            "orion_get_client_waits": ([I, ctypes.POINTER(ctypes.c_ulonglong), I], I),
            "orion_trace_start": ([], None), "orion_trace_end": ([ctypes.c_char_p], I),
        }
        for name, (args, res) in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res

    def __getattr__(self, name):
        return getattr(self.lib, name)

    def waits(self, client: int, reset: bool = False) -> dict:
        out = (ctypes.c_ulonglong * 8)()
        self.lib.orion_get_client_waits(client, out, 1 if reset else 0)
        return {"waits": int(out[0]), "total_ms": out[1] / 1e6, "max_ms": out[2] / 1e6,
                "max_op": int(out[3]), "max_queued_ms": out[4] / 1e6,
                "max_exec_ms": out[5] / 1e6, "max_bytes": int(out[6])}

    def stats(self, client: int) -> dict:
        out = (ctypes.c_ulonglong * 6)()
        self.lib.orion_get_client_stats(client, out)
        keys = ("ops", "kx_ops", "passthrough_ops", "be_blocked", "yields", "errors")
        d = dict(zip(keys, (int(v) for v in out)))
        d["host_holds"] = int(self.lib.orion_get_client_host_holds(client))
        return d


def preloaded() -> bool:
    """True when libgpu_scheduler.so is in LD_PRELOAD of this process."""
    return os.path.basename(LIBSHIM) in os.environ.get("LD_PRELOAD", "")


def preload_env(extra: dict | None = None) -> dict:
    env = dict(os.environ)
    pre = env.get("LD_PRELOAD", "")
    if os.path.basename(LIBSHIM) not in pre:
        env["LD_PRELOAD"] = (LIBSHIM + (":" + pre if pre else ""))
    if extra:
        env.update(extra)
    return env


# -------------------------------------------------------------- workloads ---

def make_gpt(vocab=32000, emb=512, head_size=64, layers=6, seq=256, device="cuda",
             dtype=None, dropout=0.4):
    """The reference's CharGPT (python/GPT.py:27-149) at the given sizes: per-head
    q/k/v projections (MaskedAttention) concatenated and projected, GELU FFN,
    pre-LayerNorm blocks, learned positions, dropout 0.4 on the attention
    weights, after the projection and after the FFN (active in training
    only).  Linear and embedding weights N(0, 0.02), biases zero."""
    import torch
    import torch.nn as nn
    import torch.nn.functional as F

    class Head(nn.Module):  # GPT.py:44-67
        def __init__(self):
            super().__init__()
            self.key = nn.Linear(emb, head_size, bias=False)
            self.query = nn.Linear(emb, head_size, bias=False)
            self.value = nn.Linear(emb, head_size, bias=False)
            self.register_buffer("tril", torch.tril(torch.ones(seq, seq)))
            self.dropout = nn.Dropout(dropout)

        def forward(self, x):
            B, T, C = x.shape
            q, k, v = self.query(x), self.key(x), self.value(x)
            mask = self.tril[:T, :T]
            # attention(): GPT.py:27-41, scaled by the head width
            s = q @ k.transpose(-2, -1) / (q.shape[-1] ** 0.5)
            s = s.masked_fill(mask == 0, float("-inf"))
            return self.dropout(F.softmax(s, dim=-1)) @ v

    class MultiHead(nn.Module):  # GPT.py:69-88
        def __init__(self):
            super().__init__()
            self.heads = nn.ModuleList([Head() for _ in range(emb // head_size)])
            self.proj = nn.Linear(emb, emb)
            self.dropout = nn.Dropout(dropout)

        def forward(self, x):
            return self.dropout(self.proj(torch.cat([h(x) for h in self.heads], dim=-1)))

    class FeedForward(nn.Module):  # GPT.py:90-102
        def __init__(self):
            super().__init__()
            self.l1 = nn.Linear(emb, 4 * emb)
            self.l2 = nn.Linear(4 * emb, emb)
            self.dropout = nn.Dropout(dropout)

        def forward(self, x):
            return self.dropout(self.l2(F.gelu(self.l1(x))))

    class Block(nn.Module):  # GPT.py:104-119
        def __init__(self):
            super().__init__()
            self.mha = MultiHead()
            self.ff = FeedForward()
            self.ln1 = nn.LayerNorm(emb)
            self.ln2 = nn.LayerNorm(emb)

        def forward(self, x):
            x = x + self.mha(self.ln1(x))
            return x + self.ff(self.ln2(x))

    class GPT(nn.Module):  # CharGPT, GPT.py:121-149
        def __init__(self):
            super().__init__()
            self.token_embedding = nn.Embedding(vocab, emb)
            self.position_embedding = nn.Embedding(seq, emb)
            self.blocks = nn.Sequential(*[Block() for _ in range(layers)])
            self.ln = nn.LayerNorm(emb)
            self.lm_head = nn.Linear(emb, vocab)
            for m in self.modules():
                if isinstance(m, nn.Linear):
                    nn.init.normal_(m.weight, 0.0, 0.02)
                    if m.bias is not None:
                        nn.init.zeros_(m.bias)
                elif isinstance(m, nn.Embedding):
                    nn.init.normal_(m.weight, 0.0, 0.02)

        def forward(self, tokens):
            B, T = tokens.shape
            pos = torch.arange(0, T, dtype=torch.long, device=tokens.device)
            x = self.token_embedding(tokens) + self.position_embedding(pos)
            return self.lm_head(self.ln(self.blocks(x)))

    m = GPT().to(device)
    if dtype is not None:
        m = m.to(dtype)
    return m


def make_vgg16(device="cuda"):
    """torchvision VGG16 (weights=None: Kaiming-normal convolutions), the
    model the reference's VGG16Model wraps (python/VGG16.py:13-24)."""
    from torchvision.models import vgg16
    return vgg16(weights=None).to(device)


def make_llama(vocab=32000, hidden=2048, heads=16, layers=12, inter=5504, eps=1e-6,
               theta=10000.0, seq=1024, device="cuda", dtype=None):
    """The reference's CharLLaMA (python/LLaMA.py:20-98, LlamaAttention 163-208)
    at the given sizes, without grouped KV heads (kv heads = heads): RMSNorm
    x * rsqrt(mean(x^2) + eps) * w in the model's dtype, rotary embedding
    through complex multiplication with a precomputed freqs_cis buffer,
    causal masked_fill with a tril buffer, softmax in the model's dtype,
    SwiGLU MLP.  Linear and embedding weights N(0, 0.02)."""
    import torch
    import torch.nn as nn
    import torch.nn.functional as F

    hd = hidden // heads

    class RMSNorm(nn.Module):  # LLaMA.py:20-29
        def __init__(self):
            super().__init__()
            self.weight = nn.Parameter(torch.ones(hidden))

        def forward(self, x):
            rms = torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)
            return x * rms * self.weight

    def freqs_cis_table():  # precompute_freqs_cis, LLaMA.py:33-38
        freqs = 1.0 / (theta ** (torch.arange(0, hd, 2).float() / hd))
        t = torch.arange(seq).float()
        freqs = torch.outer(t, freqs)
        return torch.polar(torch.ones_like(freqs), freqs)

    def rotary(xq, xk, freqs_cis):  # apply_rotary_emb, LLaMA.py:41-47
        xq_c = torch.view_as_complex(xq.float().reshape(*xq.shape[:-1], -1, 2))
        xk_c = torch.view_as_complex(xk.float().reshape(*xk.shape[:-1], -1, 2))
        f = freqs_cis.unsqueeze(0).unsqueeze(2)
        xq_out = torch.view_as_real(xq_c * f).flatten(-2)
        xk_out = torch.view_as_real(xk_c * f).flatten(-2)
        return xq_out.type_as(xq), xk_out.type_as(xk)

    class Attn(nn.Module):  # LlamaAttention, LLaMA.py:163-208
        def __init__(self):
            super().__init__()
            self.wq = nn.Linear(hidden, hidden, bias=False)
            self.wk = nn.Linear(hidden, hidden, bias=False)
            self.wv = nn.Linear(hidden, hidden, bias=False)
            self.wo = nn.Linear(hidden, hidden, bias=False)
            self.register_buffer("freqs_cis", freqs_cis_table())
            self.register_buffer("mask", torch.tril(torch.ones(seq, seq)))

        def forward(self, x):
            B, T, _ = x.shape
            q = self.wq(x).view(B, T, heads, hd)
            k = self.wk(x).view(B, T, heads, hd)
            v = self.wv(x).view(B, T, heads, hd)
            q, k = rotary(q, k, self.freqs_cis[:T])
            q, k, v = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
            s = (q @ k.transpose(-2, -1)) / (hd ** 0.5)
            s = s.masked_fill(self.mask[:T, :T] == 0, float("-inf"))
            out = F.softmax(s, dim=-1) @ v
            return self.wo(out.transpose(1, 2).contiguous().view(B, T, -1))

    class MLP(nn.Module):  # LlamaMLP, LLaMA.py:52-60
        def __init__(self):
            super().__init__()
            self.gate_proj = nn.Linear(hidden, inter, bias=False)
            self.up_proj = nn.Linear(hidden, inter, bias=False)
            self.down_proj = nn.Linear(inter, hidden, bias=False)

        def forward(self, x):
            return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))

    class Block(nn.Module):  # LlamaBlock, LLaMA.py:63-75
        def __init__(self):
            super().__init__()
            self.attention = Attn()
            self.feed_forward = MLP()
            self.attention_norm = RMSNorm()
            self.ffn_norm = RMSNorm()

        def forward(self, x):
            x = x + self.attention(self.attention_norm(x))
            return x + self.feed_forward(self.ffn_norm(x))

    class LLaMA(nn.Module):  # CharLLaMA, LLaMA.py:78-98
        def __init__(self):
            super().__init__()
            self.token_embedding = nn.Embedding(vocab, hidden)
            self.layers = nn.Sequential(*[Block() for _ in range(layers)])
            self.norm = RMSNorm()
            self.lm_head = nn.Linear(hidden, vocab, bias=False)
            for m in self.modules():
                if isinstance(m, (nn.Linear, nn.Embedding)):
                    nn.init.normal_(m.weight, 0.0, 0.02)

        def forward(self, tokens):
            x = self.layers(self.token_embedding(tokens))
            return self.lm_head(self.norm(x))

    m = LLaMA().to(device)
    if dtype is not None:
        m = m.to(dtype)
    return m


def gpt_flops_forward(batch, seq=256, emb=512, layers=6, vocab=32000, ffn=2048):
    """Captured-GEMM FLOPs of one forward of the 6-layer d512 GPT."""
    tok = batch * seq
    per_layer = (2 * tok * emb * emb * 3          # q, k, v (all heads)
                 + 2 * batch * seq * seq * emb * 2  # scores + att@v (all heads)
                 + 2 * tok * emb * emb            # proj
                 + 2 * tok * emb * ffn * 2)       # l1 + l2
    return layers * per_layer + 2 * tok * emb * vocab


def vgg16_flops_forward(batch):
    """Conv + FC FLOPs of one VGG16 forward at 224x224."""
    cfg = [(3, 64, 224), (64, 64, 224), (64, 128, 112), (128, 128, 112), (128, 256, 56),
           (256, 256, 56), (256, 256, 56), (256, 512, 28), (512, 512, 28), (512, 512, 28),
           (512, 512, 14), (512, 512, 14), (512, 512, 14)]
    conv = sum(2 * batch * ci * co * 9 * hw * hw for ci, co, hw in cfg)
    fc = 2 * batch * (25088 * 4096 + 4096 * 4096 + 4096 * 1000)
    return conv + fc


# ------------------------------------------------------------ client loop ---

class ClientResult:
    def __init__(self):
        self.latencies_ms: list[float] = []
        # host wall time the client thread spent issuing each step (the step's
        # Python and enqueue work, including waits for the GIL)
        self.issue_ms: list[float] = []
        self.iters = 0
        self.elapsed_ms = 0.0
        self.error: BaseException | None = None


def write_trace(orion: Orion, path: str) -> int:
    """Ends the interposer's capture trace and writes it to path (gzip when the
    path ends in .gz).  Returns the number of events."""
    import gzip
    import shutil
    import tempfile
    if not path.endswith(".gz"):
        return orion.orion_trace_end(path.encode())
    fd, tmp = tempfile.mkstemp(suffix=".json")
    os.close(fd)
    try:
        n = orion.orion_trace_end(tmp.encode())
        with open(tmp, "rb") as src, gzip.open(path, "wb") as dst:
            shutil.copyfileobj(src, dst)
    finally:
        os.unlink(tmp)
    return n


def percentile(xs, q):
    if not xs:
        return float("nan")
    s = sorted(xs)
    k = (len(s) - 1) * q
    f = math.floor(k)
    c = min(f + 1, len(s) - 1)
    return s[f] + (s[c] - s[f]) * (k - f)


_client_streams: dict = {}
_streams_lock = threading.Lock()


def client_stream(dev: int, client: int):
    """The stream client `client` issues its work on, on device `dev`: one per
    client for the life of the process, so every phase of a run reuses it
    (per-stream state such as the kx scratch buffers is then made once).  The
    HP client's stream has the device's highest priority, so the hardware
    schedules its blocks ahead of BE blocks waiting for the same SMs."""
    import torch
    with _streams_lock:
        key = (dev, client)
        if key not in _client_streams:
            _client_streams[key] = torch.cuda.Stream(device=dev, priority=-1 if client == 0 else 0)
        return _client_streams[key]


def run_clients(orion: Orion | None, hp_step, be_step, hp_steps: int, hp_warmup: int,
                be_warmup: int = 1, with_be: bool = True, with_hp: bool = True,
                be_seconds: float | None = None, hp_period_ms: float = 0.0,
                on_start=None):
    """Runs the HP loop (hp_warmup + hp_steps timed iterations, CUDA events per
    iteration in the HP client's stream order) and, concurrently, the BE
    loop(s) until HP finishes (or for be_seconds when HP is off).  Client
    identity: HP = 0, BE = 1, 2, ... registered on each thread as the
    reference drivers do.  be_step is one step function or a list of them
    (one BE client each); the BE result is returned in the same form.
    on_start, when given, runs once in the HP thread after every client
    finished its warm-up, before HP's last warm-up step, which runs beside
    the BE loops and flows into the timed steps without a synchronisation
    (or at the start barrier when there is no HP loop)."""
    import torch

    be_steps = list(be_step) if isinstance(be_step, (list, tuple)) else [be_step]
    if not with_be:
        be_steps = []
    hp_res = ClientResult()
    be_res = [ClientResult() for _ in be_steps]
    # CUDA's current device is per thread and a new thread starts on device 0:
    # the client threads adopt the caller's device before creating streams
    dev = torch.cuda.current_device()
    stop = threading.Event()
    parties = (1 if with_hp else 0) + len(be_steps)
    # on_start runs in the HP thread right before its first timed step (after
    # its warm-up), or as the start barrier's action when there is no HP loop
    ready = threading.Barrier(max(1, parties), action=None if with_hp else on_start)

    def hp_thread():
        try:
            torch.cuda.set_device(dev)
            s = client_stream(dev, 0)
            if orion is not None:
                orion.orion_set_client_idx(0)
                orion.orion_register_client_stream(0, ctypes.c_void_p(s.cuda_stream))
            with torch.cuda.stream(s):
                # the last warm-up step runs after the start barrier, beside the
                # BE clients' loops, so the first timed step is not the first
                # one HP issues against them
                pre = hp_warmup - 1 if hp_warmup > 1 and be_steps else hp_warmup
                for _ in range(pre):
                    hp_step()
                # torch creates a CUDA event at its first record, and creating
                # one can block the thread for milliseconds (the driver grows its
                # event pool): create all timing events before the timed loop
                evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                       for _ in range(hp_steps)]
                first = torch.cuda.Event(enable_timing=True)
                last = torch.cuda.Event(enable_timing=True)
                for ev in [first, last] + [e for pair in evs for e in pair]:
                    ev.record(s)
                s.synchronize()
                ready.wait()
                if on_start is not None:
                    on_start()
                # no synchronisation between this warm-up step and the timed
                # ones: an idle gap would let the scheduler lower the HP flag
                # and the BE clients' queued work take the GPU just as the
                # first timed step starts
                for _ in range(hp_warmup - pre):
                    hp_step()
                first.record(s)
                for a, b in evs:
                    t_issue = time.perf_counter()
                    a.record(s)
                    hp_step()
                    b.record(s)
                    hp_res.issue_ms.append((time.perf_counter() - t_issue) * 1e3)
                    if hp_period_ms > 0:
                        while (time.perf_counter() - t_issue) * 1e3 < hp_period_ms:
                            time.sleep(0.0002)
                last.record(s)
                s.synchronize()
                hp_res.latencies_ms = [a.elapsed_time(b) for a, b in evs]
                hp_res.elapsed_ms = first.elapsed_time(last)
                hp_res.iters = hp_steps
        except BaseException as e:  # noqa: BLE001 - reported by the caller
            hp_res.error = e
            ready.abort()
        finally:
            stop.set()
            if orion is not None:
                orion.orion_set_client_idx(-1)

    def be_thread(i):
        res, step, client = be_res[i], be_steps[i], i + 1
        try:
            torch.cuda.set_device(dev)
            s = client_stream(dev, client)
            if orion is not None:
                orion.orion_set_client_idx(client)
                orion.orion_register_client_stream(client, ctypes.c_void_p(s.cuda_stream))
            with torch.cuda.stream(s):
                for _ in range(be_warmup):
                    step()
                s.synchronize()
                ready.wait()
                start = torch.cuda.Event(enable_timing=True)
                end = torch.cuda.Event(enable_timing=True)
                start.record(s)
                t0 = time.perf_counter()
                n = 0
                while True:
                    step()
                    n += 1
                    if with_hp and stop.is_set():
                        break
                    if not with_hp and be_seconds is not None and time.perf_counter() - t0 >= be_seconds:
                        break
                end.record(s)
                s.synchronize()
                res.iters = n
                res.elapsed_ms = start.elapsed_time(end)
        except BaseException as e:  # noqa: BLE001
            res.error = e
            ready.abort()
        finally:
            if orion is not None:
                orion.orion_set_client_idx(-1)

    threads = []
    if with_hp:
        threads.append(threading.Thread(target=hp_thread, name="HP-Client"))
    for i in range(len(be_steps)):
        threads.append(threading.Thread(target=be_thread, args=(i,), name=f"BE{i + 1}-Client"))
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    for r in [hp_res] + be_res:
        if r.error is not None and not isinstance(r.error, threading.BrokenBarrierError):
            raise r.error
    for r in [hp_res] + be_res:
        if r.error is not None:
            raise r.error
    if isinstance(be_step, (list, tuple)):
        return hp_res, be_res
    return hp_res, (be_res[0] if be_res else ClientResult())
