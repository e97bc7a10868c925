"""Torch-facing wrappers of the sm_100a task operators.

Each function takes CUDA tensors laid out as the task's OpSpec declares (row-major,
contiguous), allocates the output if none is given, and enqueues the kernel on the current
torch CUDA stream through the C ABI.  There is no fallback: a CPU tensor, a wrong dtype or a
missing native library raises.
"""

from __future__ import annotations

import functools

import torch

from . import _native

_TORCH_DTYPES = {torch.float16: "fp16", torch.bfloat16: "bf16", torch.float32: "fp32", torch.int32: "i32"}


def dtype_name(t: torch.Tensor) -> str:
    try:
        return _TORCH_DTYPES[t.dtype]
    except KeyError as exc:
        raise TypeError(f"unsupported dtype {t.dtype}") from exc


def _check(t: torch.Tensor, name: str, dtype: torch.dtype | None = None) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (there is no CPU path)")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous (row-major)")
    if dtype is not None and t.dtype != dtype:
        raise TypeError(f"{name} has dtype {t.dtype}, expected {dtype}")


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _tensor_device(fn):
    """Run an operator on the GPU its tensors live on.

    The C ABI launches on the calling thread's current CUDA device and caches per-device state
    (SM count, kernel attributes) under it, while the stream comes from the tensors' device; so the
    call is made with that device current.  Tensors on two different GPUs are refused (a kernel
    would read the other GPU's memory); CPU tensors are left to each operator's own check, which
    refuses them."""

    @functools.wraps(fn)
    def wrapper(*args, **kwargs):
        devices = {a.device for a in (*args, *kwargs.values()) if isinstance(a, torch.Tensor) and a.is_cuda}
        if len(devices) > 1:
            raise ValueError(f"{fn.__name__}: tensors on more than one device ({', '.join(sorted(map(str, devices)))})")
        if not devices:
            return fn(*args, **kwargs)
        with torch.cuda.device(devices.pop()):
            return fn(*args, **kwargs)

    return wrapper


@_tensor_device
def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6, out: torch.Tensor | None = None) -> torch.Tensor:
    """``y = x * rsqrt(mean(x^2, -1) + eps) * w`` (tasks/rmsnorm/reference.py:110-115)."""
    _check(x, "x")
    _check(w, "w", x.dtype)
    hidden = x.shape[-1] if x.dim() else 1
    if w.numel() != hidden:
        raise ValueError(f"w has {w.numel()} elements, expected hidden={hidden}")
    rows = x.numel() // max(hidden, 1)
    if out is None:
        out = torch.empty_like(x)
    _check(out, "out", x.dtype)
    _native.call(
        "sf_rmsnorm",
        x.data_ptr(),
        w.data_ptr(),
        out.data_ptr(),
        rows,
        hidden,
        float(eps),
        _native.DTYPE_CODES[dtype_name(x)],
        _stream(x),
    )
    return out


@_tensor_device
def gemm_nt(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None, variant: int = 0) -> torch.Tensor:
    """``C = A @ B^T`` with A ``[M, K]`` and B ``[N, K]`` (fp32 accumulation, one rounding)."""
    _check(a, "A")
    _check(b, "B", a.dtype)
    if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[1]:
        raise ValueError(f"gemm_nt needs A [M,K] and B [N,K], got {tuple(a.shape)} and {tuple(b.shape)}")
    m, k = a.shape
    n = b.shape[0]
    if out is None:
        out = torch.empty((m, n), dtype=a.dtype, device=a.device)
    _check(out, "out", a.dtype)
    desc = _native.op_desc("gemm_nt", dtype_name(a), dims=(m, n, k), variant=variant)
    _native.run_op(desc, [a.data_ptr(), b.data_ptr(), out.data_ptr()], _stream(a))
    return out


@_tensor_device
def gemm_nn(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
            variant: int = 0) -> torch.Tensor:
    """``C = A @ B`` with A ``[M, K]`` and B ``[K, N]`` (tasks/gemm/reference.py:110-114).

    The tensor-core kernel reads B in place when N % 8 == 0; otherwise ``workspace`` (uint8, at
    least ``gemm_nn_workspace_bytes``, allocated here when not given) receives a transposed copy of
    B first.  Pass ``variant=2`` to force the general kernel."""
    return _gemm_kn("gemm_nn", a, b, out, workspace, variant)


@_tensor_device
def gemm_silu(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
              variant: int = 0) -> torch.Tensor:
    """``C = silu(A @ B)``, silu(v) = v * sigmoid(v) on the fp32 product (tasks/gemm_silu/reference.py,
    ``reference``).  Layouts, workspace and variants as :func:`gemm_nn`; the SiLU is fused into the
    GEMM's epilogue."""
    return _gemm_kn("gemm_silu", a, b, out, workspace, variant)


def _gemm_kn(op: str, a: torch.Tensor, b: torch.Tensor, out, workspace, variant: int) -> torch.Tensor:
    _check(a, "A")
    _check(b, "B", a.dtype)
    if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[0]:
        raise ValueError(f"{op} needs A [M,K] and B [K,N], got {tuple(a.shape)} and {tuple(b.shape)}")
    m, k = a.shape
    n = b.shape[1]
    if out is None:
        out = torch.empty((m, n), dtype=a.dtype, device=a.device)
    _check(out, "out", a.dtype)
    need = gemm_nn_workspace_bytes(m, n, k, dtype_name(a))
    if workspace is None and variant != 2 and need:
        workspace = torch.empty(need, dtype=torch.uint8, device=a.device)
    ws_ptr = workspace.data_ptr() if workspace is not None else 0
    ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    desc = _native.op_desc(op, dtype_name(a), dims=(m, n, k, ws_bytes), variant=variant)
    _native.run_op(desc, [a.data_ptr(), b.data_ptr(), out.data_ptr(), ws_ptr], _stream(a))
    return out


def gemm_nn_workspace_bytes(m: int, n: int, k: int, dtype: str) -> int:
    return int(_native.load().sf_gemm_nn_workspace_bytes(m, n, k, _native.DTYPE_CODES[dtype]))


def kernel_status(device: torch.device | None = None) -> tuple[int, int]:
    """Read and clear the tensor-core kernels' status word of ``device`` (default: the current
    device; synchronises that device's current stream)."""
    if device is None:
        return _native.kernel_status(torch.cuda.current_stream().cuda_stream)
    with torch.cuda.device(device):
        return _native.kernel_status(torch.cuda.current_stream(device).cuda_stream)


def _run(op: str, t: torch.Tensor, ptrs, dims=(), attrs=(), variant: int = 0, flags: int = 0) -> None:
    desc = _native.op_desc(op, dtype_name(t), dims=dims, attrs=attrs, variant=variant, flags=flags)
    _native.run_op(desc, ptrs, _stream(t))


@_tensor_device
def silu(x: torch.Tensor, out: torch.Tensor | None = None, variant: int = 0) -> torch.Tensor:
    """``y = x * sigmoid(x)`` (tasks/silu/reference.py:105-108), any shape, element-wise."""
    _check(x, "x")
    out = torch.empty_like(x) if out is None else out
    _check(out, "out", x.dtype)
    _run("silu", x, [x.data_ptr(), out.data_ptr()], dims=(x.numel(),), variant=variant)
    return out


@_tensor_device
def swiglu(gate: torch.Tensor, up: torch.Tensor, out: torch.Tensor | None = None, variant: int = 0) -> torch.Tensor:
    """``y = gate * sigmoid(gate) * up`` (tasks/swiglu/reference.py:109-113)."""
    _check(gate, "gate")
    _check(up, "up", gate.dtype)
    if up.numel() != gate.numel():
        raise ValueError("gate and up must have the same number of elements")
    out = torch.empty_like(gate) if out is None else out
    _check(out, "out", gate.dtype)
    _run("swiglu", gate, [gate.data_ptr(), up.data_ptr(), out.data_ptr()], dims=(gate.numel(),), variant=variant)
    return out


def _unary(op: str, x: torch.Tensor, out: torch.Tensor | None, variant: int) -> torch.Tensor:
    _check(x, "x")
    out = torch.empty_like(x) if out is None else out
    _check(out, "out", x.dtype)
    if out.numel() != x.numel():
        raise ValueError(f"{op}: out has {out.numel()} elements, x has {x.numel()}")
    _run(op, x, [x.data_ptr(), out.data_ptr()], dims=(x.numel(),), variant=variant)
    return out


@_tensor_device
def relu(x: torch.Tensor, out: torch.Tensor | None = None, variant: int = 0) -> torch.Tensor:
    """``y = max(x, 0)``; values <= 0 map to +0 and NaN propagates (tasks/relu/reference.py, ``reference``)."""
    return _unary("relu", x, out, variant)


@_tensor_device
def sigmoid(x: torch.Tensor, out: torch.Tensor | None = None, variant: int = 0) -> torch.Tensor:
    """``y = 1 / (1 + exp(-x))`` (tasks/sigmoid/reference.py, ``reference``)."""
    return _unary("sigmoid", x, out, variant)


@_tensor_device
def sigmoid_shift(x: torch.Tensor, out: torch.Tensor | None = None, variant: int = 0) -> torch.Tensor:
    """``y = sigmoid(x) + 1`` (tasks/sigmoid_shift/reference.py, ``reference``)."""
    return _unary("sigmoid_shift", x, out, variant)


@_tensor_device
def lion(p: torch.Tensor, g: torch.Tensor, m: torch.Tensor, lr: float = 1e-3, wd: float = 0.1, beta1: float = 0.9,
         beta2: float = 0.99, p_out: torch.Tensor | None = None, m_out: torch.Tensor | None = None,
         variant: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    """One Lion step (tasks/lion/reference.py, ``reference``; defaults from tasks/lion/opspec.json attrs):
    ``c = beta1*m + (1-beta1)*g``, ``p_out = p*(1 - lr*wd) - lr*sign(c)``, ``m_out = beta2*m + (1-beta2)*g``.
    Returns ``(p_out, m_out)``."""
    _check(p, "p")
    _check(g, "g", p.dtype)
    _check(m, "m", p.dtype)
    if g.numel() != p.numel() or m.numel() != p.numel():
        raise ValueError("p, g and m must have the same number of elements")
    p_out = torch.empty_like(p) if p_out is None else p_out
    m_out = torch.empty_like(p) if m_out is None else m_out
    _check(p_out, "p_out", p.dtype)
    _check(m_out, "m_out", p.dtype)
    _run("lion", p, [p.data_ptr(), g.data_ptr(), m.data_ptr(), p_out.data_ptr(), m_out.data_ptr()], dims=(p.numel(),),
         attrs=(float(lr), float(wd), float(beta1), float(beta2)), variant=variant)
    return p_out, m_out


@_tensor_device
def gemv(a: torch.Tensor, x: torch.Tensor, out: torch.Tensor | None = None, variant: int = 0) -> torch.Tensor:
    """``y[r] = sum_k A[r, k] * x[k]`` with A ``[M, K]`` row-major (tasks/gemv/reference.py, ``reference``)."""
    _check(a, "A")
    _check(x, "x", a.dtype)
    if a.dim() != 2 or x.numel() != a.shape[1]:
        raise ValueError(f"gemv needs A [M,K] and x [K], got {tuple(a.shape)} and {tuple(x.shape)}")
    m, k = a.shape
    out = torch.empty((m,), dtype=a.dtype, device=a.device) if out is None else out
    _check(out, "out", a.dtype)
    _run("gemv", a, [a.data_ptr(), x.data_ptr(), out.data_ptr()], dims=(m, k), variant=variant)
    return out


@_tensor_device
def softmax(x: torch.Tensor, out: torch.Tensor | None = None, variant: int = 0) -> torch.Tensor:
    """Row softmax over the last axis (tasks/softmax/reference.py:104-106)."""
    _check(x, "x")
    n = x.shape[-1]
    m = x.numel() // max(n, 1)
    out = torch.empty_like(x) if out is None else out
    _check(out, "out", x.dtype)
    _run("softmax", x, [x.data_ptr(), out.data_ptr()], dims=(m, n), variant=variant)
    return out


@_tensor_device
def reduction_sum(x: torch.Tensor, out: torch.Tensor | None = None, variant: int = 0) -> torch.Tensor:
    """Row sum over the last axis (tasks/reduction_sum/reference.py:104-106)."""
    _check(x, "x")
    n = x.shape[-1]
    m = x.numel() // max(n, 1)
    out = torch.empty(x.shape[:-1], dtype=x.dtype, device=x.device) if out is None else out
    _check(out, "out", x.dtype)
    _run("reduction_sum", x, [x.data_ptr(), out.data_ptr()], dims=(m, n), variant=variant)
    return out


@_tensor_device
def rope(x: torch.Tensor, base: float = 10000.0, out: torch.Tensor | None = None, variant: int = 0) -> torch.Tensor:
    """Rotate-half RoPE over ``[B, H, S, D]`` (tasks/rope/reference.py:105-115)."""
    _check(x, "x")
    if x.dim() != 4:
        raise ValueError("rope expects x [B, H, S, D]")
    b, h, s, d = x.shape
    out = torch.empty_like(x) if out is None else out
    _check(out, "out", x.dtype)
    _run("rope", x, [x.data_ptr(), out.data_ptr()], dims=(b, h, s, d), attrs=(base,), variant=variant)
    return out


@_tensor_device
def bitdelta_gemm(x: torch.Tensor, bits: torch.Tensor, scale: float = 0.02, out: torch.Tensor | None = None,
                  variant: int = 0) -> torch.Tensor:
    """``y = scale * x @ W`` with W ``[K, N]`` of +-1 from ``bits [K/32, N]`` (int32/uint32 words;
    bit j of ``bits[kb, n]`` is ``W[kb*32 + j, n]``, set = +1) — tasks/bitdelta_gemm/reference.py:99-130."""
    _check(x, "x")
    _check(bits, "bits")
    if bits.element_size() != 4:
        raise TypeError("bits must hold 32-bit words")
    m, k = x.shape
    kb, n = bits.shape
    if kb * 32 != k:
        raise ValueError(f"bits has {kb} word rows, expected K/32 = {k // 32}")
    out = torch.empty((m, n), dtype=x.dtype, device=x.device) if out is None else out
    _check(out, "out", x.dtype)
    _run("bitdelta_gemm", x, [x.data_ptr(), bits.data_ptr(), out.data_ptr()], dims=(m, n, k), attrs=(scale,), variant=variant)
    return out


@_tensor_device
def bitdelta_gemm_base(x: torch.Tensor, w_base: torch.Tensor, s_words: torch.Tensor, alpha: torch.Tensor,
                       out: torch.Tensor | None = None, variant: int = 0) -> torch.Tensor:
    """``y = x @ (W_base + diag(alpha) S)^T`` with S in {-1,+1} packed along K as ``s_words [N, K/32]``."""
    _check(x, "x")
    _check(w_base, "w_base", x.dtype)
    _check(s_words, "s_words")
    _check(alpha, "alpha", x.dtype)
    m, k = x.shape
    n = w_base.shape[0]
    if w_base.shape[1] != k or s_words.shape != (n, k // 32) or alpha.numel() != n:
        raise ValueError("bitdelta_gemm_base: inconsistent shapes")
    out = torch.empty((m, n), dtype=x.dtype, device=x.device) if out is None else out
    _check(out, "out", x.dtype)
    _run("bitdelta_gemm_base", x, [x.data_ptr(), w_base.data_ptr(), s_words.data_ptr(), alpha.data_ptr(), out.data_ptr()],
         dims=(m, n, k), variant=variant)
    return out


@_tensor_device
def flash_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float, causal: bool = False,
                    out: torch.Tensor | None = None, variant: int = 0) -> torch.Tensor:
    """``softmax(q k^T * scale [+ causal mask]) v`` over ``[B, H, S, D]``
    (tasks/flash_attention/reference.py:113-119; the causal mask keeps key j <= query i)."""
    _check(q, "q")
    _check(k, "k", q.dtype)
    _check(v, "v", q.dtype)
    if q.dim() != 4 or k.shape != q.shape or v.shape != q.shape:
        raise ValueError("flash_attention expects q, k, v of the same shape [B, H, S, D]")
    b, h, s, d = q.shape
    out = torch.empty_like(q) if out is None else out
    _check(out, "out", q.dtype)
    _run("flash_attention", q, [q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr()], dims=(b, h, s, d), attrs=(scale,),
         variant=variant, flags=1 if causal else 0)
    return out


@_tensor_device
def varlen_kda(q, k, v, g, beta, a_log, dt_bias, initial_state, cu_seqlens, scale, lower_bound: float = -5.0,
               output: torch.Tensor | None = None, final_state: torch.Tensor | None = None, variant: int = 0,
               workspace: torch.Tensor | None = None):
    """Packed-varlen KDA forward (tasks/varlen_kda/reference.py:323-374).  ``scale`` is the
    task's one-element fp32 tensor; returns ``(output [T,H,D], final_state [N,H,D,D])``.
    ``variant``: 0 = the two-pass kernels over ``workspace`` (uint8, at least
    ``varlen_kda_workspace_bytes``; allocated here when not given) where they apply (D = 128),
    else the 16-token chunked kernel (D = 128), else the recurrent one; 4 = two-pass only;
    1 = 16-token chunked only; 2 = recurrent only."""
    for name, t in (("q", q), ("k", k), ("v", v), ("g", g), ("beta", beta)):
        _check(t, name, q.dtype)
    for name, t in (("A_log", a_log), ("dt_bias", dt_bias), ("initial_state", initial_state), ("scale", scale)):
        _check(t, name, torch.float32)
    _check(cu_seqlens, "cu_seqlens", torch.int32)
    t_, h, d = q.shape
    n = cu_seqlens.numel() - 1
    output = torch.empty_like(v) if output is None else output
    final_state = torch.empty((n, h, d, d), dtype=torch.float32, device=q.device) if final_state is None else final_state
    need = varlen_kda_workspace_bytes(t_, n, h, d) if variant in (0, 4) and n > 0 else 0
    if workspace is None and need:
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    ws_ptr = workspace.data_ptr() if workspace is not None else 0
    ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    ptrs = [x.data_ptr() for x in (q, k, v, g, beta, a_log, dt_bias, initial_state, cu_seqlens, scale, output, final_state)]
    _run("varlen_kda", q, ptrs + [ws_ptr], dims=(n, h, d, t_, ws_bytes), attrs=(lower_bound,), variant=variant)
    return output, final_state


def varlen_kda_workspace_bytes(total_tokens: int, num_seqs: int, heads: int, dim: int) -> int:
    """Workspace bytes of the two-pass varlen KDA kernels (0 when they do not apply)."""
    return int(_native.load().sf_varlen_kda_workspace_bytes(total_tokens, num_seqs, heads, dim))


@_tensor_device
def kda(q, k, v, g, beta, a_log, dt_bias, initial_state, scale, lower_bound: float = -5.0,
        output: torch.Tensor | None = None, final_state: torch.Tensor | None = None,
        work_items: torch.Tensor | None = None, item_counts: torch.Tensor | None = None,
        handoff_states: torch.Tensor | None = None, variant: int = 0):
    """Fixed-length KDA forward (tasks/kda/reference.py ``reference``): the varlen recurrence over
    one sequence of N tokens.  q, k, v, g ``[N, H, D]``, beta ``[N, H]``; A_log ``[H]``, dt_bias
    ``[H*D]``, initial_state ``[H, D, D]`` and the one-element ``scale`` in fp32.  The task's
    candidate-owned outputs (``work_items`` u32 ``[3, 2]`` as int32, ``item_counts`` ``[1]``,
    ``handoff_states`` ``[2, H, D, D]``) are allocated when not given; the work list is written,
    the hand-off states are not (one piece).  ``variant`` 0/2 run the recurrent fp32 kernel (the
    default at every D), 1 forces the chunked tensor-core kernel (D = 128).  Returns
    ``(output [N,H,D], final_state [H,D,D])``."""
    for name, t in (("q", q), ("k", k), ("v", v), ("g", g), ("beta", beta)):
        _check(t, name, q.dtype)
    for name, t in (("A_log", a_log), ("dt_bias", dt_bias), ("initial_state", initial_state), ("scale", scale)):
        _check(t, name, torch.float32)
    n, h, d = q.shape
    dev = q.device
    output = torch.empty_like(v) if output is None else output
    final_state = torch.empty((h, d, d), dtype=torch.float32, device=dev) if final_state is None else final_state
    work_items = torch.empty((3, 2), dtype=torch.int32, device=dev) if work_items is None else work_items
    item_counts = torch.empty((1,), dtype=torch.int32, device=dev) if item_counts is None else item_counts
    handoff_states = torch.empty((2, h, d, d), dtype=torch.float32, device=dev) if handoff_states is None else handoff_states
    ptrs = [x.data_ptr() for x in (q, k, v, g, beta, a_log, dt_bias, initial_state, scale, output, final_state, work_items,
                                   item_counts, handoff_states)]
    _run("kda", q, ptrs, dims=(n, h, d), attrs=(lower_bound,), variant=variant)
    return output, final_state


@_tensor_device
def varlen_kda_gated(q, k, v, g, beta, cu_seqlens, scale: float, initial_state: torch.Tensor | None = None,
                     output: torch.Tensor | None = None, final_state: torch.Tensor | None = None, variant: int = 0,
                     workspace: torch.Tensor | None = None):
    """Gated KDA workload: q, k pre-normalised, ``g`` fp32 log-decay used directly, ``beta`` fp32
    gate used directly, state from zero (or ``initial_state``).

    At D = 128 the default (and ``variant=4``) runs the two-pass kernels over ``workspace`` (uint8,
    at least ``varlen_kda_gated_workspace_bytes``; allocated here when not given); ``variant=1``
    forces the single-pass 32-token kernel, 2 the recurrent kernel, 3 the 16-token kernel."""
    for name, t in (("q", q), ("k", k), ("v", v)):
        _check(t, name, q.dtype)
    _check(g, "g", torch.float32)
    _check(beta, "beta", torch.float32)
    _check(cu_seqlens, "cu_seqlens", torch.int32)
    t_, h, d = q.shape
    n = cu_seqlens.numel() - 1
    output = torch.empty_like(v) if output is None else output
    final_state = torch.empty((n, h, d, d), dtype=torch.float32, device=q.device) if final_state is None else final_state
    s0 = 0
    if initial_state is not None:
        _check(initial_state, "initial_state", torch.float32)
        s0 = initial_state.data_ptr()
    need = varlen_kda_gated_workspace_bytes(t_, n, h, d) if variant in (0, 4) else 0
    if workspace is None and need:
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    ws_ptr = workspace.data_ptr() if workspace is not None else 0
    ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    ptrs = [q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(), beta.data_ptr(), cu_seqlens.data_ptr(), s0,
            output.data_ptr(), final_state.data_ptr(), ws_ptr]
    _run("varlen_kda_gated", q, ptrs, dims=(n, h, d, t_, ws_bytes), attrs=(scale,), variant=variant)
    return output, final_state


def varlen_kda_gated_workspace_bytes(total_tokens: int, num_seqs: int, heads: int, dim: int) -> int:
    """Workspace bytes of the two-pass gated KDA kernels (0 when they do not apply)."""
    return int(_native.load().sf_varlen_kda_gated_workspace_bytes(total_tokens, num_seqs, heads, dim))


@_tensor_device
def mamba2_chunk_scan(x, dt, dA_cumsum, b_mat, c_mat, d_skip, states, out: torch.Tensor | None = None,
                      variant: int = 0) -> torch.Tensor:
    """Mamba-2 SSD chunk scan of one B/C group (tasks/mamba2_chunk_scan/reference.py:106-127).

    x [B,L,H,P], dt [B,L,H], dA_cumsum [B,H,NC,CHUNK], b_mat/c_mat [B,L,N], d_skip [H],
    states [B,NC,H,P,N], all of one 16-bit dtype; returns y [B,L,H,P]."""
    tensors = (("x", x), ("dt", dt), ("dA_cumsum", dA_cumsum), ("Bmat", b_mat), ("Cmat", c_mat), ("Dskip", d_skip),
               ("states", states))
    for name, t in tensors:
        _check(t, name, x.dtype)
    if x.dim() != 4 or dA_cumsum.dim() != 4 or states.dim() != 5:
        raise ValueError("mamba2_chunk_scan expects x [B,L,H,P], dA_cumsum [B,H,NC,CHUNK], states [B,NC,H,P,N]")
    bsz, seq, heads, hd = x.shape
    nc, chunk = dA_cumsum.shape[2], dA_cumsum.shape[3]
    n = b_mat.shape[-1]
    want = {"dt": (bsz, seq, heads), "dA_cumsum": (bsz, heads, nc, chunk), "Bmat": (bsz, seq, n), "Cmat": (bsz, seq, n),
            "Dskip": (heads,), "states": (bsz, nc, heads, hd, n)}
    for name, t in tensors[1:]:
        if tuple(t.shape) != want[name]:
            raise ValueError(f"{name} has shape {tuple(t.shape)}, expected {want[name]}")
    if nc * chunk != seq:
        raise ValueError(f"SEQLEN {seq} != NCHUNKS {nc} * CHUNK {chunk}")
    out = torch.empty_like(x) if out is None else out
    _check(out, "out", x.dtype)
    ptrs = [t.data_ptr() for _, t in tensors] + [out.data_ptr()]
    _run("mamba2_chunk_scan", x, ptrs, dims=(bsz, seq, heads, hd, n, chunk), variant=variant)
    return out
