"""The reference operator itself, run on the GPU box from its prebuilt kernels — TEST INFRASTRUCTURE.

xCalibur's operator (kernels/moe_w4a16_h200/moe_w4a16.py, "moe.py" below) is Python over one CUDA kernel that it
compiles at run time.  ``oracle/build_ref.py`` compiles that kernel, from the reference's own sources and through
its own build path, into ``oracle/_ref/okc_*.so`` in a container that has the reference; the GPU box has only
those modules.  This file restates, in torch, the host side that the modules need there:

* ``prepare`` (moe.py:3292-3351): the lossless repacks of the weights into the kernel's layouts — mma-fragment
  code words with the GF(2) word transform (``_pack_codes`` + ``_xc_transform_words``, moe.py:3168-3181,
  :3903-3933), scale bytes (``_pack_scales``, :3184-3191), the fat order (:3194-3201) and the unit order
  (:3204-3209) — the e4m3 -> bf16 x 2^64 LUT (:3313-3318) and the scratch (``_make_scratch``, :3353-3367);
* ``kernel_fn`` (moe.py:3370-3399 and the M = 1 wrapper at :3956-3969): the build picked by token count M and the
  384-token chunk loop around ``okc_run``.

The restated packers are pinned bit for bit against the reference's own packers (digests of their outputs on
seeded inputs, made by ``tests/golden/make_golden.py`` in a container with the reference, checked by
``tests/test_okc_pack.py``); the GF(2) transform's column table is the reference's ``_XC_COLS``, read from the
committed fixture ``tests/golden/ref_gf2.json`` that the same script extracted.

Only tests and ``bench.py``'s reference arm use this module.  The operator is shape-locked: H = I = 4096, 256
experts, 32 local experts starting at expert 0, top-8 (moe.py:105-110).
"""
from __future__ import annotations

import importlib.machinery
import importlib.util
import json
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
GOLDEN = os.path.join(os.path.dirname(HERE), "tests", "golden")

# the reference's fixed model shape (moe.py:105-110) and per-call chunk bound (moe.py:115-117)
HIDDEN = 4096
TOP_K = 8
N_EXPERTS_TOTAL = 256
LOCAL_START = 0
LOCAL_EXPERTS = 32
CHUNK_TOKENS = 384
EMAX = CHUNK_TOKENS * TOP_K
# stream-K fixup area and activation rows of the WGS build, which only size the scratch here (moe.py:119-125)
WGS_SLOTS, WGS_FIXW = 160, 4096
WGS_FIXF = 2 * WGS_SLOTS * 4 * WGS_FIXW + 2 * WGS_SLOTS * 4 + 136 * 16
WGS_XROWS = EMAX + 8 * (32 + EMAX // 32 + 8)

# the token-count bounds of the builds kernel_fn picks (moe.py:131-153); M = 1 runs the program build
TINY_MAX_M, TINY2_MAX_M, MID_MAX_M = 4, 8, 16


class Unavailable(RuntimeError):
    """The reference's kernel cannot run here (not built, or one CTA per SM does not fit)."""


# ------------------------------------------------------------------------------------------------ layouts
def _code_bit_targets():
    """(register, upper half, code bit) -> bit of the packed word before the GF(2) transform.

    Register r of a word feeds four bf16x2 fragments; a code's bits (m, e0, e1, s) sit at bf16 bits 6, 7, 8, 15
    (+16 in the upper half) after the register's rotation in the DQ7 decoder (moe.py:3123-3146): the word is read
    as stored (r = 0), shifted by 4 (r = 1), rotated by 10 (r = 2) and shifted by 6 with e1 rotated by 14 (r = 3),
    so the stored bit is the output bit plus (0, 28, 22, 26 / 18) mod 32."""
    out = {}
    field = (6, 7, 8, 15)
    for reg in range(4):
        for half in range(2):
            for bit in range(4):
                shift = (0, 28, 22, 26)[reg] if not (reg == 3 and bit == 2) else 18
                out[(reg, half, bit)] = (field[bit] + 16 * half + shift) % 32
    assert sorted(out.values()) == list(range(32))
    return out


_TARGETS = _code_bit_targets()
# register r of a word holds (row half h, first k j0) = (0,0) (1,0) (0,2) (1,2) of its 16-row x 4-k group
_REG_ROWHALF_K = ((0, 0), (1, 0), (0, 2), (1, 2))


def gate_up_rows(I: int, device=None) -> torch.Tensor:
    """Packed row order of gate_up: 8 gate rows, then the 8 matching up rows, and so on (moe.py:3303-3305)."""
    blk = torch.arange(I // 8, device=device)[:, None] * 8 + torch.arange(8, device=device)[None, :]
    return torch.stack((blk, blk + I), dim=1).reshape(-1)


def _xc_cols():
    with open(os.path.join(GOLDEN, "ref_gf2.json")) as f:
        return [int(v) for v in json.load(f)["xc_cols"]]


def gf2_transform(words: torch.Tensor, cols) -> torch.Tensor:
    """Apply the reference's word transform: bit i of the input contributes column cols[i] (XOR)."""
    w = words.to(torch.int64) & 0xFFFFFFFF
    out = torch.zeros_like(w)
    for i, c in enumerate(cols):
        out ^= ((w >> i) & 1) * int(c)
    return torch.where(out >= 2**31, out - 2**32, out).to(torch.int32)


def pack_code_words(codes: torch.Tensor, rows: torch.Tensor, cols) -> torch.Tensor:
    """codes uint8 [R0, 2048] (one expert, K = 4096, low nibble = even k) in row order `rows` -> int32 words in
    the order [16-row block][warp 8][chunk 8][g 8][t 4][step 4]; each word holds, for register r, the codes of
    row 16 rb + 8 h + g at k = 512 w + 64 c + 16 t + 4 s + j0 + {0, 1} ((h, j0) from _REG_ROWHALF_K)."""
    dev = codes.device
    c = codes.index_select(0, rows.to(dev))
    R = c.shape[0]
    nib = torch.stack((c & 0xF, c >> 4), dim=-1).reshape(R, -1).to(torch.int64)  # [R, 4096]
    nb = R // 16
    ar = lambda n: torch.arange(n, device=dev)
    rb = ar(nb).view(nb, 1, 1, 1, 1, 1)
    w = ar(8).view(1, 8, 1, 1, 1, 1)
    ch = ar(8).view(1, 1, 8, 1, 1, 1)
    g = ar(8).view(1, 1, 1, 8, 1, 1)
    t = ar(4).view(1, 1, 1, 1, 4, 1)
    s = ar(4).view(1, 1, 1, 1, 1, 4)
    kbase = 512 * w + 64 * ch + 16 * t + 4 * s
    word = torch.zeros((nb, 8, 8, 8, 4, 4), dtype=torch.int64, device=dev)
    for reg, (h, j0) in enumerate(_REG_ROWHALF_K):
        row = 16 * rb + 8 * h + g
        for half in range(2):
            code = nib[row, kbase + j0 + half]
            for bit in range(4):
                word |= ((code >> bit) & 1) << _TARGETS[(reg, half, bit)]
    word = torch.where(word >= 2**31, word - 2**32, word).to(torch.int32).reshape(-1)
    return gf2_transform(word, cols)


def pack_scale_bytes(sf: torch.Tensor, rows: torch.Tensor) -> torch.Tensor:
    """E4M3 scale bytes [R0, 256] in row order `rows` -> bytes [16-row block][warp 8][g 8][t 4][chunk 8][h 2]:
    the scale of row 16 rb + 8 h + g for k block 32 w + 4 c + t."""
    dev = sf.device
    s = sf.contiguous().view(torch.uint8).index_select(0, rows.to(dev))
    nb = s.shape[0] // 16
    ar = lambda n: torch.arange(n, device=dev)
    rb = ar(nb).view(nb, 1, 1, 1, 1, 1)
    w = ar(8).view(1, 8, 1, 1, 1, 1)
    g = ar(8).view(1, 1, 8, 1, 1, 1)
    t = ar(4).view(1, 1, 1, 4, 1, 1)
    ch = ar(8).view(1, 1, 1, 1, 8, 1)
    h = ar(2).view(1, 1, 1, 1, 1, 2)
    return s[16 * rb + 8 * h + g, 32 * w + 4 * ch + t].reshape(-1).contiguous()


def fat_order(words: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """One expert's code words and scale bytes -> [256-row unit][k stage of 256 (16)][36864 B]: 32 KB of codes
    [16-row block][chunk of the stage 4][lane 32][16 B], then 4 KB of scales [16-row block][lane][chunk 4][h 2]."""
    nu = words.numel() // (16 * 8 * 8 * 32 * 4)
    # words: [unit][rb16][w][chunk-half][chunk 4][lane][4]; stage = (w, chunk-half)
    cw = words.view(nu, 16, 8, 2, 4, 32, 4).permute(0, 2, 3, 1, 4, 5, 6).contiguous()
    cb = cw.view(torch.uint8).view(nu, 16, 32768)
    # scales: [unit][rb16][w][lane][chunk-half][chunk 4][h]
    sb = scales.view(nu, 16, 8, 32, 2, 4, 2).permute(0, 2, 4, 1, 3, 5, 6).contiguous().view(nu, 16, 4096)
    return torch.cat((cb, sb), dim=2).reshape(-1).contiguous()


def unit_order(words: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """One expert -> per 16-row block its 32 KB of code words, then its 4 KB of scale bytes."""
    nb = words.numel() // (8 * 8 * 32 * 4)
    return torch.cat((words.contiguous().view(torch.uint8).view(nb, 32768), scales.contiguous().view(nb, 4096)),
                     dim=1).reshape(-1).contiguous()


def e4m3_lut(device) -> torch.Tensor:
    """E4M3 byte -> bf16(value * 2^64) in both halves of an int32 (moe.py:3313-3318)."""
    v = torch.arange(256, dtype=torch.int32, device=device).to(torch.uint8).view(torch.float8_e4m3fn).float()
    b = (v * 2.0**64).to(torch.bfloat16).view(torch.int16).to(torch.int32) & 0xFFFF
    return (b | (b << 16)).to(torch.int32).contiguous()


def scales_prmt_exact(*sfs) -> bool:
    """Every scale byte is a positive normal E4M3 value (0x08..0x7E): the condition under which the reference uses
    its PRMT scale decode, the build compiled here (moe.py:3109-3116)."""
    for sf in sfs:
        b = sf.contiguous().view(torch.uint8)
        if bool(((b < 0x08) | (b > 0x7E)).any()):
            return False
    return True


# ------------------------------------------------------------------------------------------------ the operator
def prepare(weights, device=None) -> dict:
    """The reference's ``prepare`` (moe.py:3292-3351) for its 32 local experts, without compiling anything: the
    packed layouts in the order ``okc_run`` reads them (moe.py:2812-2820), the LUT, the scratch and the grid."""
    dev = device or weights["w13"].device
    lo, cnt = LOCAL_START, LOCAL_EXPERTS
    I = weights["w13"].shape[1] // 2
    H = weights["w2"].shape[1]
    if I != HIDDEN or H != HIDDEN:
        raise Unavailable(f"the reference is built for H = I = {HIDDEN}, got H = {H}, I = {I}")
    if not scales_prmt_exact(weights["w13_sf"][lo:lo + cnt], weights["w2_sf"][lo:lo + cnt]):
        raise Unavailable("scale bytes outside 0x08..0x7E: the reference would use its LUT build (not built here)")
    cols = _xc_cols()
    rows_a = gate_up_rows(I, dev)
    rows_b = torch.arange(H, device=dev)
    wa, sa, wb, sb, fa, fb, ua, ub = ([] for _ in range(8))
    for e in range(lo, lo + cnt):
        c13 = weights["w13"][e].to(dev).contiguous().view(torch.uint8) ^ 0x88   # sign fold (moe.py:3311)
        a_w = pack_code_words(c13, rows_a, cols)
        a_s = pack_scale_bytes(weights["w13_sf"][e].to(dev), rows_a)
        b_w = pack_code_words(weights["w2"][e].to(dev).contiguous().view(torch.uint8), rows_b, cols)
        b_s = pack_scale_bytes(weights["w2_sf"][e].to(dev), rows_b)
        wa.append(a_w), sa.append(a_s), wb.append(b_w), sb.append(b_s)
        fa.append(fat_order(a_w, a_s)), fb.append(fat_order(b_w, b_s))
        ua.append(unit_order(a_w, a_s)), ub.append(unit_order(b_w, b_s))
    f32 = lambda t: t.to(device=dev, dtype=torch.float32).contiguous()
    w = [torch.cat(wa), torch.cat(sa), f32(weights["w13_gs"][lo:lo + cnt]),
         torch.cat(wb), torch.cat(sb), f32(weights["w2_gs"][lo:lo + cnt]),
         e4m3_lut(dev), weights["post_norm_w"].to(dev).contiguous(),
         torch.cat(fa), torch.cat(fb), torch.cat(ua), torch.cat(ub)]
    scratch = [torch.zeros(8 + 1024 + EMAX, dtype=torch.int32, device=dev),
               torch.zeros(EMAX + EMAX * HIDDEN + WGS_FIXF, dtype=torch.float32, device=dev),
               torch.zeros((EMAX + 2 * WGS_XROWS) * HIDDEN, dtype=torch.bfloat16, device=dev)]
    grid = torch.cuda.get_device_properties(dev).multi_processor_count
    return {"w": w, "lo": lo, "cnt": cnt, "scratch": scratch, "grid": grid}


_MODULES: dict = {}


def manifest() -> dict:
    path = os.path.join(REF_DIR, "manifest.json")
    if not os.path.exists(path):
        raise Unavailable("oracle/_ref/manifest.json is missing: run oracle/build_ref.py where the reference is")
    with open(path) as f:
        return json.load(f)


def module(build: str):
    """The built extension module of one reference build, loaded once and admitted: the reference's own
    admission routine must find one CTA per SM resident (its grid barrier needs every CTA of the grid)."""
    if build in _MODULES:
        return _MODULES[build]
    info = manifest()["builds"].get(build)
    if info is None:
        raise Unavailable(f"reference build {build!r} was not built")
    path = os.path.join(REF_DIR, info["so"])
    loader = importlib.machinery.ExtensionFileLoader(info["module"], path)
    spec = importlib.util.spec_from_file_location(info["module"], path, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    adm = int(mod.xc_admission())
    if adm < 1:
        raise Unavailable(f"reference build {build!r}: one CTA per SM does not fit (admission {adm})")
    mod.okc_set_pdl(0)                      # the reference's default (PDL = False, moe.py:169)
    _MODULES[build] = mod
    return mod


def build_for(M: int) -> str:
    """The build kernel_fn runs for M tokens (moe.py:3384-3393, :3956-3969); the WGS MAIN build, which needs
    wgmma, is replaced by its mma.sync fallback (the only substitution)."""
    if M == 1:
        return "program"
    if M <= TINY_MAX_M:
        return "tiny"
    if M <= TINY2_MAX_M:
        return "tiny2"
    if M <= MID_MAX_M:
        return "mid"
    return "main"


def kernel_fn(data, state) -> torch.Tensor:
    """The reference's ``kernel_fn`` (moe.py:3370-3399): fresh output, ids as int32 (16-byte aligned), weights as
    fp32, launched in 384-token chunks on the current stream."""
    cfg = data["config"]
    x = data["hidden_states"].contiguous()
    M = x.shape[0]
    if cfg["local_start"] != state["lo"] or cfg["local_count"] != state["cnt"]:
        raise ValueError("config local range differs from the prepared state")
    ids = data["topk_ids"].to(torch.int32).contiguous()
    if ids.data_ptr() & 15:
        ids = ids.clone()
    tw = data["topk_weights"].to(torch.float32).contiguous()
    out = torch.empty((M, HIDDEN), dtype=torch.bfloat16, device=x.device)
    ext = module(build_for(M))
    for m0 in range(0, M, CHUNK_TOKENS):
        m1 = min(M, m0 + CHUNK_TOKENS)
        ext.okc_run(state["w"], state["scratch"], x[m0:m1], ids[m0:m1], tw[m0:m1], out[m0:m1], state["lo"],
                    state["cnt"], state["grid"])
    return out
