"""Generate golden vectors from the reference's own Triton kernels.

Run in a container that has the reference package mounted (read-only), its
root given by ``--ref`` or the ``TMO_REFERENCE_ROOT`` environment variable::

    TRITON_INTERPRET=1 python tests/golden/make_golden.py --ref <reference package root>

The reference cannot be imported as a package here (it needs ``torch_mlu``
and Cambricon's Triton backend), so this script loads its kernel files by
path under the Triton CPU interpreter with three shims, and copies no
reference source into this repository:

* ``torch_mlu_ops.triton.utils.get_total_core_num`` -> a constant core count;
* ``device="mlu"`` allocations -> CPU tensors;
* the package names ``torch_mlu_ops.triton.fla.*`` -> the files by path.

The chunk path additionally needs two substitutions that the Cambricon
toolchain provides and upstream Triton lacks (see ``_load_chunk_modules``).
Outputs: ``*.npz`` files next to this script with inputs and outputs.
"""

from __future__ import annotations

import argparse
import importlib.util
import os
import sys
import types
import zlib

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))


def _install_shims(ref: str):
    pkg = types.ModuleType("torch_mlu_ops")
    pkg.__path__ = [ref]
    sys.modules["torch_mlu_ops"] = pkg
    tri = types.ModuleType("torch_mlu_ops.triton")
    tri.__path__ = [os.path.join(ref, "triton")]
    sys.modules["torch_mlu_ops.triton"] = tri
    fla = types.ModuleType("torch_mlu_ops.triton.fla")
    fla.__path__ = [os.path.join(ref, "triton", "fla")]
    sys.modules["torch_mlu_ops.triton.fla"] = fla
    utils = types.ModuleType("torch_mlu_ops.triton.utils")
    utils.get_total_core_num = lambda: 8
    sys.modules["torch_mlu_ops.triton.utils"] = utils

    # "mlu" device requests become CPU allocations.
    def _cpu(kw):
        if str(kw.get("device", "")) == "mlu":
            kw["device"] = "cpu"
        return kw

    for name in ("empty_like", "empty", "zeros"):
        orig = getattr(torch, name)

        def wrap(*a, _orig=orig, **kw):
            return _orig(*a, **_cpu(kw))
        setattr(torch, name, wrap)
    orig_new_empty = torch.Tensor.new_empty
    torch.Tensor.new_empty = lambda self, *a, **kw: orig_new_empty(self, *a, **_cpu(kw))


def _load(modname: str, path: str, source_patch=None):
    if source_patch is None:
        spec = importlib.util.spec_from_file_location(modname, path)
        mod = importlib.util.module_from_spec(spec)
        sys.modules[modname] = mod
        spec.loader.exec_module(mod)
        return mod
    with open(path) as f:
        src = f.read()
    src = source_patch(src)
    mod = types.ModuleType(modname)
    mod.__file__ = path
    sys.modules[modname] = mod
    # Triton's interpreter reads kernel source through inspect/linecache:
    # register the in-memory text under the module's file name.
    import linecache
    fake = path + ".interp"
    linecache.cache[fake] = (len(src), None, src.splitlines(True), fake)
    exec(compile(src, fake, "exec"), mod.__dict__)
    return mod


def _rng_inputs(seed, B, T, H, HV, K, V, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, H, K, generator=g).to(dtype)
    k = torch.randn(B, T, H, K, generator=g).to(dtype)
    v = torch.randn(B, T, HV, V, generator=g).to(dtype)
    gg = torch.nn.functional.logsigmoid(torch.randn(B, T, HV, generator=g))
    beta = torch.sigmoid(torch.randn(B, T, HV, generator=g))
    return q, k, v, gg, beta, g


def _np(x):
    return None if x is None else x.detach().float().numpy() if x.dtype != torch.int64 else x.numpy()


def gen_recurrent_fn(ref: str):
    """Decode kernel with a V-first slot cache (``fused_recurrent_fn.py``)."""
    mod = _load("torch_mlu_ops.triton.fla.fused_recurrent_fn",
                os.path.join(ref, "triton/fla/fused_recurrent_fn.py"))
    cases = []
    # (name, N, T, H, HV, K, V, l2norm, spec, inplace, pad, beta_per_v)
    cases.append(("decode_basic", 6, 1, 2, 4, 16, 16, True, False, True, True, False))
    cases.append(("decode_nonorm_betav", 5, 1, 2, 2, 16, 8, False, False, True, False, True))
    cases.append(("decode_spec", 4, 3, 1, 2, 8, 16, True, True, True, True, False))
    cases.append(("decode_notinplace", 3, 1, 2, 4, 16, 16, True, False, False, False, False))
    for (name, N, T, H, HV, K, V, l2, spec, inplace, pad, bpv) in cases:
        q, k, v, gg, beta, gen = _rng_inputs(zlib.crc32(name.encode()) % 1000, 1, N * T, H, HV, K, V)
        if bpv:
            beta = torch.sigmoid(torch.randn(1, N * T, HV, V, generator=gen))
        slots = 3 * N + 2
        cache = torch.randn(slots, HV, V, K, generator=gen) * 0.5
        cu = torch.arange(0, N * T + 1, T, dtype=torch.int64)
        perm = torch.randperm(slots, generator=gen)
        idx = perm[: N * max(T, 1)].reshape(N, T).clone() if inplace else perm[:N].clone()
        if pad:
            idx[1, 0] = -1
        nacc = None
        if spec:
            # the initial state is read from column nacc-1 of each index row
            nacc = torch.randint(1, T + 1, (N,), generator=gen)
        cache_in = cache.clone()
        o, ht = mod.fused_recurrent_gated_delta_rule(
            q, k, v, gg, beta, 0.37, cache, inplace_final_state=inplace, cu_seqlens=cu,
            ssm_state_indices=idx, num_accepted_tokens=nacc, use_qk_l2norm_in_kernel=l2)
        np.savez_compressed(
            os.path.join(HERE, f"rfn_{name}.npz"),
            q=_np(q), k=_np(k), v=_np(v), g=_np(gg), beta=_np(beta), scale=np.float64(0.37),
            cache_in=_np(cache_in), cu_seqlens=cu.numpy(), ssm_state_indices=idx.numpy(),
            num_accepted_tokens=(nacc.numpy() if nacc is not None else np.zeros(0, np.int64)),
            l2norm=np.bool_(l2), inplace=np.bool_(inplace), o=_np(o), final_state=_np(ht))
        print("wrote", name)


def gen_recurrent_fn_kda(ref: str):
    """The decode kernel's per-key decay branch (``IS_KDA``,
    ``fused_recurrent_fn.py:77-80,115-120``).  The reference facade always
    passes ``IS_KDA=False`` (``:230``), so the kernel is launched here
    directly, with the launch arguments its host wrapper builds (``:161-233``)
    and ``g`` holding per-key log decays ``[B, T, HV, K]``."""
    mod = sys.modules.get("torch_mlu_ops.triton.fla.fused_recurrent_fn") or _load(
        "torch_mlu_ops.triton.fla.fused_recurrent_fn", os.path.join(ref, "triton/fla/fused_recurrent_fn.py"))
    import triton
    # (name, N, T, H, HV, K, V, l2norm, pad)
    cases = [("decode_kda", 5, 2, 2, 4, 16, 16, True, True)]
    for (name, N, T, H, HV, K, V, l2, pad) in cases:
        q, k, v, _, beta, gen = _rng_inputs(zlib.crc32(name.encode()) % 1000, 1, N * T, H, HV, K, V)
        gk = torch.nn.functional.logsigmoid(torch.randn(1, N * T, HV, K, generator=gen)) * 0.5
        slots = 3 * N + 2
        cache = torch.randn(slots, HV, V, K, generator=gen) * 0.5
        cu = torch.arange(0, N * T + 1, T, dtype=torch.int64)
        idx = torch.randperm(slots, generator=gen)[: N * T].reshape(N, T).clone()
        if pad:
            idx[1, 0] = -1
        cache_in = cache.clone()
        o = torch.empty_like(v)
        BK, BV = triton.next_power_of_2(K), min(8, triton.next_power_of_2(V))
        sis, sit = idx.stride()
        mod.tmo_fused_recurrent_gated_delta_rule_fwd_kernel[(triton.cdiv(V, BV), N * HV)](
            q=q, k=k, v=v, g=gk, beta=beta, o=o, h0=cache, ht=cache, cu_seqlens=cu,
            ssm_state_indices=idx, num_accepted_tokens=None, scale=0.29, N=N, T=N * T, B=1, H=H, HV=HV,
            K=K, V=V, BK=BK, BV=BV, stride_init_state_token=cache.stride(0),
            stride_final_state_token=cache.stride(0), stride_indices_seq=sis, stride_indices_tok=sit,
            IS_BETA_HEADWISE=False, USE_QK_L2NORM_IN_KERNEL=l2, INPLACE_FINAL_STATE=True, IS_KDA=True,
            num_warps=1, num_stages=3)
        np.savez_compressed(
            os.path.join(HERE, f"rfn_{name}.npz"),
            q=_np(q), k=_np(k), v=_np(v), g=_np(gk), beta=_np(beta), scale=np.float64(0.29),
            cache_in=_np(cache_in), cu_seqlens=cu.numpy(), ssm_state_indices=idx.numpy(),
            num_accepted_tokens=np.zeros(0, np.int64), l2norm=np.bool_(l2), inplace=np.bool_(True),
            o=_np(o), final_state=_np(cache))
        print("wrote", name)


def gen_recurrent(ref: str):
    """Plain K-first recurrence (``fused_recurrent.py``), incl. config 0 shape."""
    mod = _load("torch_mlu_ops.triton.fla.fused_recurrent",
                os.path.join(ref, "triton/fla/fused_recurrent.py"))
    # (name, B, T, H, HV, K, V, l2norm, varlen, h0)
    cases = [("plain_gva", 1, 37, 2, 4, 16, 16, True, False, True),
             ("plain_varlen", 1, 50, 2, 2, 16, 8, False, True, True),
             ("cfg0_t64", 1, 64, 4, 4, 64, 64, True, False, False)]
    for (name, B, T, H, HV, K, V, l2, varlen, use_h0) in cases:
        q, k, v, gg, beta, gen = _rng_inputs(zlib.crc32(name.encode()) % 1000 + 7, B, T, H, HV, K, V)
        cu = torch.tensor([0, 11, 11, 30, T], dtype=torch.int64) if varlen else None
        N = B if cu is None else len(cu) - 1
        h0 = torch.randn(N, HV, K, V, generator=gen) * 0.3 if use_h0 else None
        o, ht = mod.fused_recurrent_gated_delta_rule_fwd(
            q, k, v, g=gg, beta=beta, scale=K ** -0.5, initial_state=h0,
            output_final_state=True, use_qk_l2norm_in_kernel=l2, cu_seqlens=cu)
        np.savez_compressed(
            os.path.join(HERE, f"rec_{name}.npz"),
            q=_np(q), k=_np(k), v=_np(v), g=_np(gg), beta=_np(beta), scale=np.float64(K ** -0.5),
            h0=(_np(h0) if h0 is not None else np.zeros(0, np.float32)),
            cu_seqlens=(cu.numpy() if cu is not None else np.zeros(0, np.int64)),
            l2norm=np.bool_(l2), o=_np(o), final_state=_np(ht))
        print("wrote", name)


def gen_chunk_h(ref: str):
    """The state-recurrence stage ``chunk_gated_delta_rule_fwd_h``
    (``chunk_delta_h.py:200-271``) with the per-key decay gk of its USE_GK
    branch (``:155-171``), called directly (the chunk facade never passes gk).
    The kernel's gk load covers 64 keys, so K <= 64 here; the K-first form
    needs g as well (without it the branch names a block only the g branch
    defines), so gk alone is taken with the V-first state."""
    _load_chunk_modules(ref)
    mod = sys.modules["torch_mlu_ops.triton.fla.chunk_delta_h"]
    # (name, T, Hg, H, K, V, use_g, state_v_first, varlen)
    cases = [("h_g_gk", 150, 2, 4, 32, 16, True, False, False),
             ("h_gk_vfirst", 130, 1, 2, 64, 32, False, True, False),
             ("h_g_gk_varlen_vfirst", 200, 2, 2, 32, 16, True, True, True)]
    for (name, T, Hg, H, K, V, use_g, vfirst, varlen) in cases:
        gen = torch.Generator().manual_seed(zlib.crc32(name.encode()) % 1000 + 21)
        k = torch.nn.functional.normalize(torch.randn(1, T, Hg, K, generator=gen), dim=-1)
        w = torch.randn(1, T, H, K, generator=gen) * 0.3
        u = torch.randn(1, T, H, V, generator=gen)
        cu = torch.tensor([0, 64, 90, T], dtype=torch.int64) if varlen else None
        bounds = [(0, T)] if cu is None else [(int(cu[i]), int(cu[i + 1])) for i in range(len(cu) - 1)]

        def chunk_cumsum(x):  # chunk-local cumsum along T (dim 1) of every sequence
            out = torch.zeros_like(x)
            for bos, eos in bounds:
                for s0 in range(bos, eos, 64):
                    e0 = min(s0 + 64, eos)
                    out[:, s0:e0] = torch.cumsum(x[:, s0:e0], dim=1)
            return out

        g = chunk_cumsum(torch.nn.functional.logsigmoid(torch.randn(1, T, H, generator=gen)))
        gk = chunk_cumsum(torch.nn.functional.logsigmoid(torch.randn(1, T, H, K, generator=gen)) * 0.2)
        g_hm = g.permute(2, 0, 1).contiguous() if use_g else None  # head-major, as chunk.py:32 passes it
        N = len(bounds)
        h0 = torch.randn((N, H, V, K) if vfirst else (N, H, K, V), generator=gen) * 0.3
        h, v_new, ht = mod.chunk_gated_delta_rule_fwd_h(
            k=k, w=w, u=u, g=g_hm, gk=gk, initial_state=h0, output_final_state=True,
            state_v_first=vfirst, cu_seqlens=cu, allow_tf32=False)
        np.savez_compressed(
            os.path.join(HERE, f"chh_{name}.npz"),
            k=_np(k), w=_np(w), u=_np(u), g=_np(g_hm) if use_g else np.zeros(0, np.float32), gk=_np(gk),
            h0=_np(h0), cu_seqlens=(cu.numpy() if cu is not None else np.zeros(0, np.int64)),
            state_v_first=np.bool_(vfirst), h=_np(h), v_new=_np(v_new), final_state=_np(ht))
        print("wrote", name)


def _load_chunk_modules(ref: str):
    """Load the chunk-path kernels.  Two substitutions are needed to run them
    on upstream Triton: the Cambricon-only integer row indexing of a register
    block in the KK^T kernel is expressed as a masked row reduction, and the
    absent native ``torch_mlu_ops.solve_tril`` is served by the same file's
    own Triton merge kernel (``solve_tril.py``'s ``merge_16x16_to_64x64``
    path, which the reference keeps as its non-native implementation)."""
    _load("torch_mlu_ops.triton.fla.utils", os.path.join(ref, "triton/fla/utils.py"))
    _load("torch_mlu_ops.triton.fla.index", os.path.join(ref, "triton/fla/index.py"))
    _load("torch_mlu_ops.triton.fla.op", os.path.join(ref, "triton/fla/op.py"))

    def cumsum_patch(src):
        return "import warnings\n" + src

    _load("torch_mlu_ops.triton.fla.cumsum", os.path.join(ref, "triton/fla/cumsum.py"), cumsum_patch)

    def kkt_patch(src):
        row = "tl.sum(tl.where(tl.arange(0, H)[:, None] == id_h, {0}, 0), 0)"
        src = src.replace("b_beta[id_h,:]", row.format("b_beta"))
        src = src.replace("b_g[id_h,:]", row.format("b_g"))
        return src

    _load("torch_mlu_ops.triton.fla.chunk_scaled_dot_kkt",
          os.path.join(ref, "triton/fla/chunk_scaled_dot_kkt.py"), kkt_patch)
    st = _load("torch_mlu_ops.triton.fla.solve_tril", os.path.join(ref, "triton/fla/solve_tril.py"))
    for m in ("wy_fast", "chunk_delta_h", "chunk_o"):
        _load(f"torch_mlu_ops.triton.fla.{m}", os.path.join(ref, f"triton/fla/{m}.py"))
    return st


def gen_chunk(ref: str):
    st = _load_chunk_modules(ref)
    names = [n for n in dir(st) if "merge_16x16_to_64x64" in n]
    if not names:
        print("solve_tril merge kernel not found; chunk fixtures skipped")
        return
    merge = getattr(st, names[0])

    def native_solve_tril(A, output, cu_seqlens):
        # The merge kernel stores only the 16x16 blocks that hold valid rows;
        # the native op returns a full block (zeros outside the triangle), so
        # clear the output first.
        import triton
        output.zero_()
        B, T, H, BT = A.shape
        index = sys.modules["torch_mlu_ops.triton.fla.index"]
        ci = index.prepare_chunk_indices(cu_seqlens, BT) if cu_seqlens is not None else None
        NT = triton.cdiv(T, BT) if cu_seqlens is None else len(ci)
        merge[NT, B * H](A=A, Ai=output, cu_seqlens=cu_seqlens, chunk_indices=ci, T=T, H=H, BT=BT,
              USE_TMA=False, DOT_PRECISION="ieee")

    torch.ops.torch_mlu_ops = types.SimpleNamespace(solve_tril=native_solve_tril)
    chunk = _load("torch_mlu_ops.triton.fla.chunk", os.path.join(ref, "triton/fla/chunk.py"))
    # H == HV only: the reference KK^T kernel indexes k by v-head (see oracle).
    cases = [("chunk_t130", 1, 130, 2, 2, 32, 32, False, True),
             ("chunk_varlen", 1, 200, 2, 2, 32, 16, True, True)]
    for (name, B, T, H, HV, K, V, varlen, use_h0) in cases:
        q, k, v, gg, beta, gen = _rng_inputs(zlib.crc32(name.encode()) % 1000 + 11, B, T, H, HV, K, V)
        q = torch.nn.functional.normalize(q, dim=-1)
        k = torch.nn.functional.normalize(k, dim=-1)
        cu = torch.tensor([0, 64, 90, T], dtype=torch.int64) if varlen else None
        N = B if cu is None else len(cu) - 1
        h0 = torch.randn(N, HV, K, V, generator=gen) * 0.3 if use_h0 else None
        o, ht, *_ = chunk.chunk_gated_delta_rule_fwd(
            q, k, v, gg, beta, K ** -0.5, h0, True, cu_seqlens=cu, allow_tf32=False)
        np.savez_compressed(
            os.path.join(HERE, f"chk_{name}.npz"),
            q=_np(q), k=_np(k), v=_np(v), g=_np(gg), beta=_np(beta), scale=np.float64(K ** -0.5),
            h0=(_np(h0) if h0 is not None else np.zeros(0, np.float32)),
            cu_seqlens=(cu.numpy() if cu is not None else np.zeros(0, np.int64)),
            o=_np(o), final_state=_np(ht))
        print("wrote", name)


def gen_chunk_bwd(ref: str):
    """Backward fixtures from ``chunk_gated_delta_rule_bwd`` (``chunk.py:76-186``).

    Under the interpreter the backward kernels need two more changes: their
    autotune lists are cut to the first config (the interpreter cannot time
    configs), and two Cambricon-only forms are rewritten: a row of a
    ones-vector product taken with ``[0, :]`` becomes the equivalent row
    reduction, and the ``[0, :]`` of a [1, BT] block before a store becomes a
    reshape."""
    import re

    import triton
    orig_autotune = triton.autotune
    triton.autotune = lambda configs, key, **kw: orig_autotune(configs[:1], key, **kw)
    orig_load = _load

    def bwd_patch(src):
        src = re.sub(r"tl\.dot\((\w+)_ones_vec, tl\.trans\((.*?)\), allow_tf32=False\)\[0,\s*:\]",
                     r"tl.sum(\2, axis=1)", src)
        return src.replace("b_dg.to(p_dg.dtype.element_ty)[0,:]",
                           "tl.reshape(b_dg.to(p_dg.dtype.element_ty), (BT,))")

    def load_patched(modname, path, source_patch=None):
        def patch(src):
            return bwd_patch(source_patch(src) if source_patch is not None else src)
        return orig_load(modname, path, patch)

    globals()["_load"] = load_patched
    try:
        st = _load_chunk_modules(ref)
        merge = getattr(st, [n for n in dir(st) if "merge_16x16_to_64x64" in n][0])

        def native_solve_tril(A, output, cu_seqlens):
            output.zero_()
            B, T, H, BT = A.shape
            index = sys.modules["torch_mlu_ops.triton.fla.index"]
            ci = index.prepare_chunk_indices(cu_seqlens, BT) if cu_seqlens is not None else None
            NT = triton.cdiv(T, BT) if cu_seqlens is None else len(ci)
            merge[NT, B * H](A=A, Ai=output, cu_seqlens=cu_seqlens, chunk_indices=ci, T=T, H=H, BT=BT,
                  USE_TMA=False, DOT_PRECISION="ieee")

        torch.ops.torch_mlu_ops = types.SimpleNamespace(solve_tril=native_solve_tril)
        chunk = _load("torch_mlu_ops.triton.fla.chunk", os.path.join(ref, "triton/fla/chunk.py"))
        # (name, B, T, H, K, V, cu_seqlens, h0, dht); H == HV as in gen_chunk
        cases = [("t130", 1, 130, 2, 32, 32, None, True, True),
                 ("varlen", 1, 200, 2, 32, 16, [0, 64, 90, 200], True, True),
                 ("batch_nostate", 2, 71, 1, 16, 32, None, False, False)]
        for (name, B, T, H, K, V, cu_l, use_h0, use_dht) in cases:
            q, k, v, gg, beta, gen = _rng_inputs(zlib.crc32(name.encode()) % 1000 + 31, B, T, H, H, K, V)
            q = torch.nn.functional.normalize(q, dim=-1)
            k = torch.nn.functional.normalize(k, dim=-1)
            cu = torch.tensor(cu_l, dtype=torch.int64) if cu_l is not None else None
            N = B if cu is None else len(cu) - 1
            h0 = torch.randn(N, H, K, V, generator=gen) * 0.3 if use_h0 else None
            scale = K ** -0.5
            o, ht, A, gcum, _ = chunk.chunk_gated_delta_rule_fwd(
                q, k, v, gg, beta, scale, h0, True, cu_seqlens=cu, allow_tf32=False)
            do = torch.randn(o.shape, generator=gen)
            # the reference's dh kernel reads dht unconditionally (its zero
            # initialisation is commented out, chunk_delta_h.py:338): pass zeros
            dht = torch.randn(ht.shape, generator=gen) if use_dht else torch.zeros(ht.shape)
            dq, dk, dv, db, dg, dh0 = chunk.chunk_gated_delta_rule_bwd(
                q, k, v, gcum, beta, A, scale, h0, do, dht, cu_seqlens=cu, allow_tf32=False)
            empty = np.zeros(0, np.float32)
            np.savez_compressed(
                os.path.join(HERE, f"bwd_{name}.npz"),
                q=_np(q), k=_np(k), v=_np(v), g=_np(gg), beta=_np(beta), scale=np.float64(scale),
                h0=_np(h0) if h0 is not None else empty,
                cu_seqlens=cu.numpy() if cu is not None else np.zeros(0, np.int64),
                do=_np(do), dht=_np(dht) if dht is not None else empty,
                dq=_np(dq), dk=_np(dk), dv=_np(dv), db=_np(db), dg=_np(dg),
                dh0=_np(dh0) if (dh0 is not None and h0 is not None) else empty)
            print("wrote bwd", name)
    finally:
        triton.autotune = orig_autotune
        globals()["_load"] = orig_load


def _load_conv_modules(ref: str):
    """Load ``triton/conv`` by path.  Four substitutions: the fla forward
    launcher passes a Cambricon compiler option (``bottleneck=``) that
    upstream Triton does not accept, which is dropped; the autotune lists
    keep one block size each, since the interpreter has no device to
    benchmark configurations on (the block size only tiles the channels);
    and the fla forward's no-initial-state branch, which loads one
    (BT + W - 1)-row block and slices it per tap (a non-power-of-2 block and
    register slicing, both Cambricon extensions), is expressed as the same
    kernel's per-tap block loads from its initial-state branch
    (``kernels.py:114-122``): the same sum over taps of shifted rows; the
    vLLM launcher's metadata grid callback no longer writes its (identical)
    program tables back into the launch arguments."""
    _load("torch_mlu_ops.triton.fla.utils", os.path.join(ref, "triton/fla/utils.py"))
    _load("torch_mlu_ops.triton.fla.index", os.path.join(ref, "triton/fla/index.py"))
    conv = types.ModuleType("torch_mlu_ops.triton.conv")
    conv.__path__ = [os.path.join(ref, "triton", "conv")]
    sys.modules["torch_mlu_ops.triton.conv"] = conv

    def kernels_patch(src):
        src = src.replace("for BD in [128, 256]", "for BD in [128]").replace(
            "for num_stages in [2,4]", "for num_stages in [2]")
        head = "        if not USE_INITIAL_STATE:\n"
        tail = "        elif i_t * BT >= W:\n"
        i, j = src.index(head), src.index(tail)
        per_tap = (head +
                   "            for i_w in tl.static_range(-W + 1, 1):\n"
                   "                p_yi = tl.make_block_ptr(p_x, (T, D), (stride_x_t, stride_x_d), "
                   "(i_t * BT + i_w, i_d * BD), (BT, BD), (1, 0))\n"
                   "                b_yi = tl.load(p_yi, boundary_check=(0, 1)).to(tl.float32)\n"
                   "                if HAS_WEIGHT:\n"
                   "                    b_yi *= tl.sum(b_w * (o_w == (i_w + W - 1)), 1)\n"
                   "                b_y += b_yi\n")
        return src[:i] + per_tap + src[j:]

    _load("torch_mlu_ops.triton.conv.kernels", os.path.join(ref, "triton/conv/kernels.py"), kernels_patch)

    def ops_patch(src):
        # (the metadata grid callback re-assigns the program tables into the
        # launch arguments; under the interpreter that replaces the converted
        # pointers with raw tensors, so the re-assignment of the very same
        # tensors is dropped)
        src = src.replace('bottleneck="simd",', "")
        src = src.replace('META["batch_ptr"] = nums_dict', '_same_table = nums_dict')
        return src.replace('META["token_chunk_offset_ptr"] = nums_dict', '_same_table = nums_dict')

    return _load("torch_mlu_ops.triton.conv.ops", os.path.join(ref, "triton/conv/ops.py"), ops_patch)


def gen_conv(ref: str):
    """Causal conv1d: the fla forward, the vLLM forward with a slot cache,
    and the decode update (``triton/conv/ops.py``)."""
    ops = _load_conv_modules(ref)
    g = torch.Generator().manual_seed(zlib.crc32(b"conv") % 1000)

    # fla forward: (name, B, T, D, W, bias, residual, init, act, cu)
    fla_cases = [("fla_basic", 2, 100, 40, 4, True, True, False, "silu", None),
                 ("fla_init", 2, 70, 24, 3, True, False, True, None, None),
                 ("fla_varlen", 1, 131, 16, 4, False, True, True, "swish", [0, 30, 31, 131])]
    for (name, B, T, D, W, hb, hr, hi, act, cu) in fla_cases:
        x = torch.randn(B, T, D, generator=g)
        w = torch.randn(D, W, generator=g) * 0.5
        b = torch.randn(D, generator=g) if hb else None
        r = torch.randn(B, T, D, generator=g) if hr else None
        cut = torch.tensor(cu, dtype=torch.int64) if cu is not None else None
        N = B if cu is None else len(cu) - 1
        h0 = torch.randn(N, D, W, generator=g) if hi else None
        y, _ = ops.causal_conv1d_fwd_fla(x, w, b, r, h0, False, act, cut)
        np.savez_compressed(os.path.join(HERE, f"conv_{name}.npz"), x=_np(x), weight=_np(w),
                            bias=_np(b) if b is not None else np.zeros(0, np.float32),
                            residual=_np(r) if r is not None else np.zeros(0, np.float32),
                            initial_state=_np(h0) if h0 is not None else np.zeros(0, np.float32),
                            cu_seqlens=np.array(cu if cu is not None else [], np.int64),
                            activation=np.str_(act or ""), y=_np(y))
        print("wrote", name)

    # vLLM forward: (name, dim, W, lens, has_init, cache_indices, lines, bias, act)
    vllm_cases = [("fn_basic", 64, 4, [5, 1, 3, 70], [1, 0, 1, 1], [3, 7, 1, 5], 8, True, "silu"),
                  ("fn_short", 48, 3, [2, 65, 1, 1], [0, 1, 1, 0], [2, 4, 6, 1], 7, False, None),
                  ("fn_null", 32, 2, [4, 9, 130], [1, 1, 0], [0, 2, 5], 6, True, "silu")]
    for (name, dim, W, lens, hin, idx, lines, hb, act) in vllm_cases:
        total = sum(lens)
        xt = torch.randn(total, dim, generator=g)       # channel-last storage
        x = xt.t()                                      # (dim, total), stride(0) == 1
        w = torch.randn(dim, W, generator=g) * 0.5
        b = torch.randn(dim, generator=g) if hb else None
        st = torch.randn(lines, W - 1, dim, generator=g)
        cs = st.transpose(1, 2)                         # (lines, dim, W-1), stride(1) == 1
        cs0 = cs.clone()
        qsl = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32)
        ci = torch.tensor(idx, dtype=torch.int32)
        hi = torch.tensor(hin, dtype=torch.bool)
        # The launcher's default path sizes its program table through
        # tensor methods that the interpreter's grid callback does not
        # expose; the reference's own ``metadata`` path takes the same table
        # precomputed (one program per 64-token block of each sequence).
        nums = [-(-n // 64) for n in lens]
        mlist = np.repeat(np.arange(len(nums)), nums).astype(np.int32)
        offs = np.concatenate([np.arange(n) for n in nums]).astype(np.int32)
        bp, tp = torch.from_numpy(mlist), torch.from_numpy(offs)
        md = types.SimpleNamespace(batch_ptr=bp, token_chunk_offset_ptr=tp, nums_dict={64: dict(
            tot=int(sum(nums)), mlist=bp, mlist_len=len(mlist), offsetlist=tp, batch_ptr=bp,
            token_chunk_offset_ptr=tp)})
        out = ops.causal_conv1d_fwd_vllm(x, w, b, cs, qsl, ci, hi, act, metadata=md)
        np.savez_compressed(os.path.join(HERE, f"conv_{name}.npz"), x=_np(x.contiguous()), weight=_np(w),
                            bias=_np(b) if b is not None else np.zeros(0, np.float32),
                            conv_states_in=_np(cs0.contiguous()), conv_states_out=_np(cs.contiguous()),
                            query_start_loc=qsl.numpy(), cache_indices=ci.numpy(), has_initial_state=hi.numpy(),
                            activation=np.str_(act or ""), out=_np(out.contiguous()))
        print("wrote", name)

    # vLLM forward with prefix caching: 2-D cache_indices, block states every
    # block_size_to_align tokens (kernels.py:254-289, :519-554)
    dim, W, lens, bsz = 32, 4, [150, 70, 10, 130], 128
    total = sum(lens)
    xt = torch.randn(total, dim, generator=g)
    x = xt.t()
    w = torch.randn(dim, W, generator=g) * 0.5
    b = torch.randn(dim, generator=g)
    lines = 16
    cs = torch.randn(lines, W - 1, dim, generator=g).transpose(1, 2)
    cs0 = cs.clone()
    qsl = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32)
    ci = torch.tensor([[1, 2, 3, 4], [5, 6, 7, 15], [8, 9, 10, 11], [12, 13, 14, 15]], dtype=torch.int32)
    first = torch.tensor([0, 1, 1, 0], dtype=torch.int32)
    last = torch.tensor([2, 2, 1, 1], dtype=torch.int32)
    init_idx = torch.tensor([0, 0, 3, 2], dtype=torch.int32)
    ncomp = torch.tensor([10, 100, 5, 64], dtype=torch.int32)  # operands of the block arithmetic stay >= 0
    hi = torch.tensor([1, 1, 0, 1], dtype=torch.bool)
    nums = [-(-n // 64) for n in lens]
    mlist = np.repeat(np.arange(len(nums)), nums).astype(np.int32)
    offs = np.concatenate([np.arange(n) for n in nums]).astype(np.int32)
    bp, tp = torch.from_numpy(mlist), torch.from_numpy(offs)
    md = types.SimpleNamespace(batch_ptr=bp, token_chunk_offset_ptr=tp, nums_dict={64: dict(
        tot=int(sum(nums)), mlist=bp, mlist_len=len(mlist), offsetlist=tp, batch_ptr=bp,
        token_chunk_offset_ptr=tp)})
    out = ops.causal_conv1d_fwd_vllm(x, w, b, cs, qsl, ci, hi, "silu", -1, 0, first, last, init_idx, ncomp,
                                     bsz, metadata=md)
    np.savez_compressed(os.path.join(HERE, "conv_fn_apc.npz"), x=_np(x.contiguous()), weight=_np(w), bias=_np(b),
                        conv_states_in=_np(cs0.contiguous()), conv_states_out=_np(cs.contiguous()),
                        query_start_loc=qsl.numpy(), cache_indices=ci.numpy(), has_initial_state=hi.numpy(),
                        block_idx_first=first.numpy(), block_idx_last=last.numpy(), initial_state_idx=init_idx.numpy(),
                        num_computed_tokens=ncomp.numpy(), block_size=np.int64(bsz), activation=np.str_("silu"),
                        out=_np(out.contiguous()))
    print("wrote fn_apc")

    # decode update: (name, N, D, W, bias, residual, act, x layout)
    upd_cases = [("upd_basic", 5, 48, 4, True, True, "silu", "nd"),
                 ("upd_w3", 3, 40, 3, False, False, None, "n1d"),
                 ("upd_1nd", 4, 16, 2, True, False, "swish", "1nd")]
    for (name, N, D, W, hb, hr, act, lay) in upd_cases:
        x2 = torch.randn(N, D, generator=g)
        x = {"nd": x2, "n1d": x2[:, None], "1nd": x2[None]}[lay]
        cache = torch.randn(N, D, W, generator=g)
        cache0 = cache.clone()
        w = torch.randn(D, W, generator=g) * 0.5
        b = torch.randn(D, generator=g) if hb else None
        r = torch.randn(N, D, generator=g) if hr else None
        y, _ = ops.causal_conv1d_update(x, cache, r, w, b, act)
        np.savez_compressed(os.path.join(HERE, f"conv_{name}.npz"), x=_np(x2), weight=_np(w),
                            bias=_np(b) if b is not None else np.zeros(0, np.float32),
                            residual=_np(r) if r is not None else np.zeros(0, np.float32),
                            cache_in=_np(cache0), cache_out=_np(cache), activation=np.str_(act or ""),
                            layout=np.str_(lay), y=_np(y.reshape(N, D)))
        print("wrote", name)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("TMO_REFERENCE_ROOT"),
                    help="root of the reference torch_mlu_ops package (read-only)")
    ap.add_argument("--only", default="")
    a = ap.parse_args()
    if not a.ref:
        ap.error("give --ref or set TMO_REFERENCE_ROOT")
    _install_shims(a.ref)
    torch.manual_seed(0)
    if a.only in ("", "rfn"):
        gen_recurrent_fn(a.ref)
    if a.only in ("", "rfn", "kda"):
        gen_recurrent_fn_kda(a.ref)
    if a.only in ("", "rec"):
        gen_recurrent(a.ref)
    if a.only in ("", "chunk"):
        gen_chunk(a.ref)
    if a.only in ("", "chunk_h"):
        gen_chunk_h(a.ref)
    if a.only in ("", "conv"):
        gen_conv(a.ref)
    if a.only in ("", "bwd"):
        gen_chunk_bwd(a.ref)


if __name__ == "__main__":
    main()
