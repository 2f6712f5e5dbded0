"""Generate the golden vectors under ``tests/golden/`` by running the reference.

This script imports the reference package (ThunderFun/convert_to_quant_QuIP_INT8,
``convert_to_quant`` v0.8.2) from a checkout given by ``--ref`` (or the
``QI8_REFERENCE_PATH`` environment variable) and executes its own code on
CPU, on seeded inputs:

* the torch CPU path (``utils/hadamard.py``, ``utils/float_utils.py``,
  ``comfy/quant_ops.py`` layouts, ``converters/quip_int8.py``), and
* its Triton kernels (``comfy/int8_kernels.py``, ``comfy/hadamard_kernels.py``)
  under the Triton CPU interpreter (``TRITON_INTERPRET=1``), so the GPU
  reference kernels' own arithmetic is pinned too.

The fixtures are small ``.npz`` files (bf16 stored as uint16 bit patterns).
They are committed; tests only read them, so nothing at test time needs the
reference.  Re-run with ``python tests/golden/make_golden.py --ref <checkout>``.
"""

import argparse
import os
import sys

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.nn.functional as F  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))


def bits(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor -> uint16 bit pattern array."""
    assert t.dtype == torch.bfloat16
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def gen(seed: int) -> torch.Generator:
    return torch.Generator(device="cpu").manual_seed(seed)


def with_outliers(x: torch.Tensor, n_ch: int, factor: float, seed: int) -> torch.Tensor:
    idx = torch.randperm(x.shape[-1], generator=gen(seed))[:n_ch]
    x = x.clone()
    x[:, idx] *= factor
    return x


def save(name: str, **arrs):
    path = os.path.join(HERE, name)
    np.savez_compressed(path, **{k: (v.numpy() if isinstance(v, torch.Tensor) else np.asarray(v))
                                 for k, v in arrs.items()})
    print(f"wrote {path} ({os.path.getsize(path)} bytes)")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("QI8_REFERENCE_PATH"),
                    required="QI8_REFERENCE_PATH" not in os.environ,
                    help="checkout of convert_to_quant (the directory holding the convert_to_quant package); "
                         "defaults to $QI8_REFERENCE_PATH")
    ap.add_argument("--only", choices=["ldlq"], default=None,
                    help="regenerate only this fixture (quip_ldlq.npz)")
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    if args.only == "ldlq":
        make_ldlq()
        return

    from convert_to_quant.utils import hadamard as H
    from convert_to_quant.utils.float_utils import quantize_int8_axiswise, quantize_int8_tensorwise
    from convert_to_quant.comfy import int8_kernels as IK
    from convert_to_quant.comfy import hadamard_kernels as HK
    from convert_to_quant.comfy.quant_ops import TensorWiseINT8Layout, AxisWiseINT8Layout
    from convert_to_quant.converters.quip_int8 import QuIPInt8Converter
    from convert_to_quant.comfy import int8_matmul_kernels as MK

    # The interpreter has no GPU to benchmark autotune candidates on; give the
    # autotuned reference kernels a single candidate (their first config) so
    # they run unchanged otherwise.  Results do not depend on the tile config.
    for k in (HK._hadamard_autotuned_stage_kernel, getattr(MK, "__mm_kernel")):
        k.configs = k.configs[:1]

    # ---------------------------------------------------------------- FWHT
    x1 = torch.randn(5, 512, generator=gen(100))
    x2 = torch.randn(3, 4096, generator=gen(101))
    x3 = torch.randn(2, 8, generator=gen(102))
    x5 = torch.randn(64, 128, generator=gen(103))
    s5r = torch.randint(0, 2, (64,), generator=gen(104)).float() * 2 - 1
    s5c = torch.randint(0, 2, (128,), generator=gen(105)).float() * 2 - 1
    save("fwht.npz",
         x1=x1, y1=H.fast_hadamard_transform(x1.clone()),
         y1n=H.fast_hadamard_transform(x1.clone(), normalize=False),
         x2=x2, y2=H.fast_hadamard_transform(x2.clone()),
         x3=x3, y3=H.fast_hadamard_transform(x3.clone()),
         x5=x5, y5_2d=H.fast_hadamard_transform_2d(x5.clone()),
         s5r=s5r, s5c=s5c,
         y5_2d_signs=HK.fast_hadamard_transform_2d_with_signs(x5.clone(), s5r, s5c),
         y5_inv_2d_signs=HK.inverse_hadamard_transform_2d_with_signs(x5.clone(), s5r, s5c, 60, 100),
         # the reference's GPU kernel, run by the Triton interpreter
         y2_triton=HK.triton_hadamard_transform(x2.clone()),
         y1_triton_signs=HK.triton_hadamard_transform_with_signs(x1.clone(), None, s5c.repeat(4)))

    # ------------------------------------------------- per-token act quant
    xa = (torch.randn(9, 3072, generator=gen(110))).to(torch.bfloat16)
    xa = with_outliers(xa.float(), 15, 30.0, 111).to(torch.bfloat16)
    xa[3].zero_()  # a zero row exercises the 1e-30 scale floor
    qa, sa = quantize_int8_axiswise(xa)
    xb = torch.randn(6, 1000, generator=gen(112)) * 3.0
    qb, sb = quantize_int8_axiswise(xb)
    save("act_token.npz", xa_bf16=bits(xa), qa=qa, sa=sa, xb=xb, qb=qb, sb=sb)

    # ------------------------------------- rotated act path (K1 composition)
    xr = with_outliers(torch.randn(7, 3072, generator=gen(120)), 40, 20.0, 121).to(torch.bfloat16)
    s_v = torch.randint(0, 2, (4096,), generator=gen(122)).float() * 2 - 1
    # quip_int8_matmul steps 1-2 (comfy/int8_kernels.py:1411-1428) on the
    # zero-padded input (converters/quip_int8.py:539-547 pad rule)
    xp = F.pad(xr.float(), (0, 4096 - 3072))
    x_had = H.fast_hadamard_transform(xp * s_v.unsqueeze(0))
    qr, sr = quantize_int8_axiswise(x_had)
    xr2 = torch.randn(5, 1024, generator=gen(123)).to(torch.bfloat16)
    s_v2 = torch.randint(0, 2, (1024,), generator=gen(124)).float() * 2 - 1
    x_had2 = H.fast_hadamard_transform(xr2.float() * s_v2.unsqueeze(0))
    qr2, sr2 = quantize_int8_axiswise(x_had2)
    save("rotate_quant.npz", x_bf16=bits(xr), s_v=s_v, x_had=x_had, q=qr, s=sr,
         x2_bf16=bits(xr2), s_v2=s_v2, x_had2=x_had2, q2=qr2, s2=sr2)

    # --------------------------------------------------- tensorwise weight
    w = (torch.randn(256, 384, generator=gen(130)) * 0.02).to(torch.bfloat16)
    qw, sw = quantize_int8_tensorwise(w)
    save("tensorwise.npz", w_bf16=bits(w), q=qw, s=sw)

    # -------------------------- Triton act/weight quant (interpreted kernels)
    xt = (torch.randn(5, 384, generator=gen(140)) * 2.0).to(torch.bfloat16)
    yt, st = IK.act_quant(xt, 128)
    xt2 = torch.randn(3, 256, generator=gen(141))
    yt2, st2 = IK.act_quant(xt2, 128)
    wt = torch.randn(256, 384, generator=gen(142)) * 0.02
    qwt, swt = IK.weight_quant(wt, 128)
    dwt = IK.weight_dequant(qwt, swt, 128, output_dtype=torch.float32)
    dat = IK.act_dequant(yt2, st2, 128, output_dtype=torch.float32)
    save("triton_quant.npz", x_bf16=bits(xt), y=yt, s=st, x2=xt2, y2=yt2, s2=st2,
         w=wt, qw=qwt, sw=swt, dw=dwt, da2=dat)

    # ----------------------------------------------------------- int32 GEMM
    ga = torch.randint(-128, 128, (37, 256), dtype=torch.int8, generator=gen(150))
    gb = torch.randint(-128, 128, (80, 256), dtype=torch.int8, generator=gen(151))
    gc = torch._int_mm(ga, gb.t().contiguous())
    gc_triton = MK.mm_8bit(ga, gb.t().contiguous())  # the reference kernel, interpreted
    assert torch.equal(gc, gc_triton)
    save("int_mm.npz", a=ga, b=gb, c=gc)

    # ----------------------------------- tensorwise / axiswise W8A8 linear
    xl = with_outliers(torch.randn(33, 512, generator=gen(160)), 5, 20.0, 161).to(torch.bfloat16)
    wl = (torch.randn(192, 512, generator=gen(162)) * 0.02).to(torch.bfloat16)
    bl = (torch.randn(192, generator=gen(163)) * 0.01).to(torch.bfloat16)
    out = {"x_bf16": bits(xl), "w_bf16": bits(wl), "bias_bf16": bits(bl)}
    for name, layout in (("tw", TensorWiseINT8Layout), ("aw", AxisWiseINT8Layout)):
        w_q, params = layout.quantize(wl)
        w_s = params["scale"]
        # optimized_linear's CUDA branch (comfy/quant_ops.py:468-474), with
        # torch._int_mm standing for mm_8bit (identical int32 semantics)
        x_q, x_s = quantize_int8_axiswise(xl.reshape(-1, xl.shape[-1]))
        res = torch._int_mm(x_q, w_q.t().contiguous())
        res_scaled = res.float() * (x_s * w_s) if w_s.ndim == 0 else res.float() * (x_s * w_s.unsqueeze(0))
        res_scaled += bl
        y = res_scaled.to(torch.bfloat16)
        out.update({f"{name}_wq": w_q, f"{name}_ws": w_s, f"{name}_xq": x_q, f"{name}_xs": x_s,
                    f"{name}_acc": res, f"{name}_y_bf16": bits(y)})
    save("linear.npz", **out)

    # --------------------------- block-K promoted GEMM (interpreted kernel)
    xg = torch.randn(64, 256, generator=gen(170)).to(torch.bfloat16)
    wg = torch.randn(256, 256, generator=gen(171)) * 0.02
    aq, a_s = IK.act_quant(xg, 128)
    bq, b_s = IK.weight_quant(wg, 128)
    bias_g = torch.randn(256, generator=gen(172)) * 0.01
    cg = IK.int8_addmm(aq, a_s, bq, b_s, bias_g)
    cg0 = IK.int8_gemm(aq, a_s, bq, b_s)
    save("gemm_block.npz", x_bf16=bits(xg), aq=aq, a_s=a_s, bq=bq, b_s=b_s, bias=bias_g,
         c_fp16=cg.view(torch.int16).numpy().view(np.uint16),
         c0_fp16=cg0.view(torch.int16).numpy().view(np.uint16))

    # ----------------------------------------------------- QuIP converter
    qc = {}
    wq = torch.randn(128, 256, generator=gen(180)) * 0.02
    common = dict(device="cpu", seed=7, actorder=False, use_diagonal_rescaling=False,
                  use_random_permutation=False)
    for tag, kw in (("row", dict(requant_scheme="tensor", requant_tensor_use_per_row_scale=True)),
                    ("glob", dict(requant_scheme="tensor", requant_tensor_use_per_row_scale=False)),
                    ("block", dict(requant_scheme="block")),
                    ("st", dict(store_transformed=True))):
        conv = QuIPInt8Converter(**common, **kw)
        res = conv.convert(wq.clone())
        qc[f"{tag}_q"] = res[0]
        qc[f"{tag}_s"] = res[1]
        if tag in ("row", "st"):
            qc[f"{tag}_deq"] = res[2]
        if tag == "st":
            qc["s_u"] = res[4]
            qc["s_v"] = res[5]
            qc["st_hsize_out"] = np.int32(res[7])
            qc["st_hsize_in"] = np.int32(res[8])
    qc["w"] = wq
    # non-power-of-two shape: the explicit composition, built from the
    # reference's own functions (converters/quip_int8.py:527-551 rotation via
    # _apply_incoherence; :1272-1274 RTN scale; :655 rounding; :1452 dequant;
    # :1489-1506 inverse; :1614-1669 requant)
    wn = torch.randn(96, 192, generator=gen(181)) * 0.02
    conv = QuIPInt8Converter(**common)
    Wp, _, _, _, s_u, s_v, _, _ = conv._apply_incoherence(wn.clone(), torch.eye(192))
    scale = (Wp.abs().amax(dim=1, keepdim=True) / 127).clamp(min=1e-12)
    Qp = torch.round(Wp / scale).clamp(-127, 127).to(torch.int8)
    Wd = Qp.to(torch.float32) * scale
    Wu = HK.fast_hadamard_transform(Wd)
    Wu = HK.fast_hadamard_transform(Wu.t()).t()
    Wu = (Wu * s_u.view(-1, 1) * s_v.view(1, -1))[:96, :192].contiguous()
    fs = (Wu.abs().amax(dim=1, keepdim=True) / 127).clamp(min=1e-12)
    Qf = torch.round(Wu / fs).clamp(-127, 127).to(torch.int8)
    Wr = Wu.view(96, 3, 64)
    bs = (Wr.abs().amax(dim=2, keepdim=True) / 127).clamp(min=1e-12)
    Qb = torch.round(Wr / bs).clamp(-127, 127).to(torch.int8).view(96, 192)
    qc.update(np_w=wn, np_s_u=s_u, np_s_v=s_v, np_wrot=Wp, np_qrot=Qp, np_srot=scale,
              np_deq=Wu, np_q_row=Qf, np_s_row=fs, np_q_block=Qb, np_s_block=bs)
    save("quip_convert.npz", **qc)

    # the converter with the reference's own defaults (act-order, diagonal
    # rescaling, random permutation and LDLQ error feedback on); the build
    # does not implement these yet, the fixture records what it must match
    qd = {}
    for tag, shape, seed in (("np", (96, 192), 182), ("p2", (128, 256), 183)):
        wd = torch.randn(*shape, generator=gen(seed)) * 0.02
        res = QuIPInt8Converter(device="cpu", seed=7).convert(wd.clone())
        qd.update({f"{tag}_w": wd, f"{tag}_q": res[0], f"{tag}_s": res[1], f"{tag}_deq": res[2]})
    save("quip_convert_defaults.npz", **qd)

    # ---------------- checkpoint format: the reference's convert_to_int8 output
    # for a tiny model (QuIP optimizer, comfy_quant metadata) in per-row
    # tensorwise, block and store-transformed modes (its --simple mode: no bias
    # correction from synthetic calibration data)
    import tempfile
    from safetensors.torch import save_file, load_file
    from convert_to_quant.quantization import convert_to_int8
    ck = {}
    gck = gen(210)
    model = {"blk.0.qkv.weight": (torch.randn(256, 128, generator=gck) * 0.02).to(torch.bfloat16),
             "blk.0.qkv.bias": (torch.randn(256, generator=gck) * 0.01).to(torch.bfloat16),
             "blk.0.proj.weight": (torch.randn(96, 192, generator=gck) * 0.02).to(torch.bfloat16),
             "norm.weight": torch.ones(128, dtype=torch.bfloat16)}

    def put(prefix, tensors):
        names = sorted(tensors)
        ck[f"{prefix}__keys"] = np.array(names)
        ck[f"{prefix}__dtypes"] = np.array([str(tensors[k].dtype).replace("torch.", "") for k in names])
        for k in names:
            v = tensors[k]
            ck[f"{prefix}/{k}"] = bits(v) if v.dtype == torch.bfloat16 else v.numpy()

    put("in", model)
    with tempfile.TemporaryDirectory() as td:
        src = os.path.join(td, "in.safetensors")
        save_file(model, src)
        for tag, kw in (("tw", {}), ("blk", {"quip_requant_scheme": "block"}),
                        ("st", {"quip_store_transformed": True})):
            dst = os.path.join(td, f"out_{tag}.safetensors")
            convert_to_int8(src, dst, comfy_quant=True, filter_flags={}, calib_samples=8, seed=0, optimizer="quip",
                            no_learned_rounding=True, quip_seed=7, quip_actorder=False, **kw)
            put(tag, load_file(dst))
    save("ckpt_quip.npz", **ck)

    # ------------- fused output requantization (interpreted Triton kernels)
    xf = torch.randn(200, 384, generator=gen(200))
    xf[:, 7] *= 25.0
    fq, fs = IK.act_quant(xf)
    wf = torch.randn(256, 384, generator=gen(201)) * 0.02
    wq_, ws_ = IK.weight_quant(wf)
    bias_f = torch.randn(256, generator=gen(202)) * 0.1
    cq, cs = IK.int8_gemm_quant(fq, fs, wq_, ws_)
    cqb, csb = IK.int8_addmm_quant(fq, fs, wq_, ws_, bias_f)
    gx = torch.randn(150, 512, generator=gen(203)) * 2.0
    gq, gs = IK.act_quant(gx)
    oq, os_ = IK.int8_gelu(gq, gs)
    save("gemm_quant.npz", aq=fq, a_s=fs, bq=wq_, b_s=ws_, bias=bias_f, c_q=cq, c_s=cs, cb_q=cqb, cb_s=csb,
         g_in_q=gq, g_in_s=gs, g_q=oq, g_s=os_)

    # -------------- GPTQ block kernel (interpreted Triton; one program per row)
    from convert_to_quant.comfy import gptq_kernels as GK
    gptq = {}
    wg = torch.randn(24, 64, generator=gen(220)) * 0.02
    xg = torch.randn(256, 64, generator=gen(221))
    hg = xg.t() @ xg / 256 + 0.01 * torch.eye(64)
    hinv = torch.linalg.cholesky(torch.cholesky_inverse(torch.linalg.cholesky(hg)), upper=True).contiguous()
    for tag, sc in (("row", (wg.abs().amax(dim=1, keepdim=True) / 127).clamp(min=1e-8)),
                    ("scalar", torch.tensor([float(wg.abs().max() / 127)]))):
        w_run = wg.clone()
        q_, e_ = GK.triton_gptq_quant_block(w_run, hinv, sc)
        gptq.update({f"{tag}_scale": sc, f"{tag}_q": q_, f"{tag}_err": e_, f"{tag}_w_out": w_run})
    save("gptq_block.npz", w=wg, hinv=hinv, **gptq)

    # ---------------------- transformed-space matmul (interpreted kernel)
    xq = torch.randn(16, 256, generator=gen(190))
    Qt = torch.randint(-127, 128, (128, 256), dtype=torch.int8, generator=gen(191))
    st_ = torch.rand(128, generator=gen(192)) * 1e-3 + 1e-4
    su = torch.randint(0, 2, (128,), generator=gen(193)).float() * 2 - 1
    sv = torch.randint(0, 2, (256,), generator=gen(194)).float() * 2 - 1
    yq = IK.quip_int8_matmul(xq, Qt, st_, su, sv)
    save("quip_matmul.npz", x=xq, Q=Qt, scale=st_, s_u=su, s_v=sv, y=yq)

    make_ldlq()


def make_ldlq():
    """The reference converter with its defaults (diagonal rescaling, random
    permutation, act-order, damping, fp64 Hessian factorization, blocked LDLQ),
    with the intermediate tensors recorded by wrapping two of its methods:
    ``_apply_incoherence`` (rescaled + rotated + permuted W and H, the signs,
    D_tilde and the random permutation) and ``_ldlq_with_iterations`` (the
    damped, act-order-permuted W, the fp32 upper Cholesky factor of H^-1 and
    the per-row scale it is given, and the Q' it returns).  The act-order
    permutation is recomputed here with the reference's own call on the damped
    diagonal.  Cases: identity Hessian at two padded widths (one block-aligned
    multi-block case) and one calibrated Hessian; per-row, block and
    store-transformed outputs."""
    from convert_to_quant.converters.quip_int8 import QuIPInt8Converter

    out = {}
    cases = (("id", (96, 192), None, {}),
             ("wide", (40, 600), None, {}),
             ("cal", (64, 160), 520, {}),
             ("blk", (96, 256), None, {"requant_scheme": "block"}),
             ("st", (80, 192), 521, {"store_transformed": True}))
    for i, (tag, shape, hseed, kw) in enumerate(cases):
        w = torch.randn(*shape, generator=gen(500 + i)) * 0.02
        w[:, 3] *= 8.0  # one outlier column, so the rescaling is not uniform
        H = None
        if hseed is not None:
            X = torch.randn(4 * shape[1], shape[1], generator=gen(hseed))
            X[:, 5] *= 4.0
            H = (X.t() @ X) / X.shape[0]
        conv = QuIPInt8Converter(device="cpu", seed=11, **kw)
        rec = {}
        inc, ldlq = conv._apply_incoherence, conv._ldlq_with_iterations

        def inc_hook(W_, H_, _f=inc, _r=rec):
            r = _f(W_, H_)
            _r.update(Wrot=r[0].clone(), Hrot=r[1].clone(), s_u=r[4], s_v=r[5],
                      D=r[6] if r[6] is not None else torch.ones(0), perm=r[7])
            return r

        def ldlq_hook(W_, Hinv_, scale_, iterations=1, _f=ldlq, _r=rec):
            _r.update(Wldlq=W_.clone(), Hinv=Hinv_.clone(), scale=scale_.clone())
            q = _f(W_, Hinv_, scale_, iterations=iterations)
            _r.update(Qldlq=q.clone())
            return q

        conv._apply_incoherence, conv._ldlq_with_iterations = inc_hook, ldlq_hook
        res = conv.convert(w.clone(), None if H is None else H.clone())
        # the act-order permutation, recomputed with the reference's own call
        Hd = rec["Hrot"].clone()
        diag = torch.diag(Hd)
        dead = diag == 0
        Hd[dead, dead] = 1
        damp = conv.percdamp * torch.mean(diag.double()).float()
        idx = torch.arange(Hd.shape[0])
        Hd[idx, idx] += damp
        order = torch.argsort(torch.diag(Hd), descending=True)
        for k in ("Hrot", "Wrot") if tag in ("id", "cal") else ("Hrot", "Hinv", "Wrot"):
            rec.pop(k)  # recomputable from pinned steps; Hinv kept for two cases
        out.update({f"{tag}_{k}": v for k, v in rec.items()})
        out.update({f"{tag}_w": w, f"{tag}_order": order, f"{tag}_damp": damp,
                    f"{tag}_q": res[0], f"{tag}_s": res[1], f"{tag}_deq": res[2]})
        if H is not None:
            out[f"{tag}_H"] = H
    save("quip_ldlq.npz", **out)


if __name__ == "__main__":
    main()
