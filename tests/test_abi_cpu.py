"""C ABI checks that need no GPU: the library loads, exports every symbol include/nk_gemm.h
declares, plans are made and validated on the host, and nk_gemm_bf16 rejects bad arguments
before touching the device."""

import ctypes
import os
import re

import pytest

import neokernel_b200 as nk
from neokernel_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    names = []
    for h in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if h.endswith(".h"):
            src = open(os.path.join(ROOT, "include", h)).read()
            names += re.findall(r"^NK_API\s+[\w\s\*]+?\b(nk_\w+)\s*\(", src, re.M)
    return names


def test_library_exports_every_declared_symbol():
    L = _lib.load()
    declared = header_functions()
    assert declared, "no NK_API declarations found"
    for name in declared:
        assert hasattr(L, name), name
    assert set(declared) == set(_lib.EXPORTS)
    assert L.nk_version() == 0x000100


def test_status_strings_distinct():
    codes = [0, -1, -2, -3, -4, -5, -6, -7, -8, -9, -10]
    texts = [_lib.status_string(c) for c in codes]
    assert len(set(texts)) == len(codes)
    assert _lib.status_string(-99) == "unknown status"


def make(M, N, K, split=0, kind=0):
    p = _lib.NkPlan()
    st = _lib.load().nk_plan_make(ctypes.byref(p), M, N, K, split, kind)
    return st, p


@pytest.mark.parametrize("args,code", [
    ((0, 16, 16), _lib.NK_ERR_SHAPE),
    ((1, 0, 16), _lib.NK_ERR_SHAPE),
    ((1, 16, 0), _lib.NK_ERR_SHAPE),
    ((1, 16, 1024, 17), _lib.NK_ERR_SPLIT),
    ((1, 16, 1024, -1), _lib.NK_ERR_SPLIT),
    ((1, 16, 1024, 0, 9), _lib.NK_ERR_ARG),
    ((1, 16, 1001, 0, _lib.KIND_GEMV), _lib.NK_ERR_ALIGN),
    ((1, 16, 1001, 2, _lib.KIND_GENERIC), _lib.NK_ERR_SPLIT),
])
def test_plan_make_rejects(args, code):
    st, p = make(*args)
    assert st == code
    assert p.magic == 0


@pytest.mark.parametrize("N,K", [(6144, 4096), (4096, 4096), (24576, 4096), (4096, 12288),
                                 (151936, 4096), (4096, 1024), (1024, 2048), (6144, 1024),
                                 (1024, 3072), (3072, 1024), (1000, 8), (7, 2056)])
@pytest.mark.parametrize("M", (1, 2, 3, 4, 8, 16, 17, 64, 256))
@pytest.mark.parametrize("split", (0, 1, 3, 16))
def test_plan_make_slices_cover_K(M, N, K, split):
    st, p = make(M, N, K, split)
    assert st == 0
    assert p.magic == _lib.PLAN_MAGIC and p.M_max == M and p.N == N and p.K == K
    if p.kind == _lib.KIND_TC:
        check_tc_partition(p, M)
        return
    assert 1 <= p.split_k <= 16
    if split:
        assert p.split_k <= split
    assert (p.split_k - 1) * p.k_slice < K <= p.split_k * p.k_slice
    assert p.k_slice % 8 == 0
    assert p.n_tiles * p.tile_n >= N and p.m_tiles * p.tile_m >= M
    ws = _lib.load().nk_ws_bytes(ctypes.byref(p))
    if p.split_k == 1:
        assert ws == 0
    else:
        assert ws >= 262144 + p.split_k * M * N * 4
        assert p.n_tiles * p.m_tiles <= 65536
        assert ws % 256 == 0


def test_forced_split_with_too_many_tiles_is_refused():
    st, p = make(16, 151936 * 16, 4096, 4, _lib.KIND_GEMV)  # 75968 tiles > 65536 tickets
    assert st == _lib.NK_ERR_SPLIT and p.magic == 0
    st, p = make(1, 151936, 4096, 4, _lib.KIND_GEMV)       # 9496 tiles fit
    assert st == 0 and p.split_k == 4


class Partition:
    """Python mirror of TcPartition (neokernel_b200/csrc/nk_common.cuh)."""

    def __init__(self, U, KB, G, split, lead=0):
        self.U, self.KB, self.G, self.split, self.lead = U, KB, G, split, lead

    def lead_units(self):
        return min(self.KB // self.split + self.lead, self.KB - (self.split - 1))

    def begin(self, c):
        if self.split == 0:
            return (self.U * c) // self.G
        t, s = divmod(c, self.split)
        if self.lead == 0 or self.split < 2 or s == 0:
            return t * self.KB + (s * self.KB) // self.split
        A = self.lead_units()
        return t * self.KB + A + ((s - 1) * (self.KB - A)) // (self.split - 1)

    def cta_of(self, u):
        if self.split == 0:
            return ((u + 1) * self.G + self.U - 1) // self.U - 1
        t, kb = divmod(u, self.KB)
        if self.lead == 0 or self.split < 2:
            return t * self.split + ((kb + 1) * self.split + self.KB - 1) // self.KB - 1
        A = self.lead_units()
        if kb < A:
            return t * self.split
        v, R = kb - A, self.KB - A
        return t * self.split + 1 + ((v + 1) * (self.split - 1) + R - 1) // R - 1


def launch_partition(p, M, aligned=False, lead=0):
    """The partition launch_tc (nk_tc.cu) builds for a call with M tokens: the tile-aligned
    one (a plan with slices, whole grid resident; its rank-0 slice `lead` K blocks longer) or
    the balanced one."""
    KB = -(-p.K // p.k_step)
    m_tiles = -(-M // p.tile_m)
    U = p.n_tiles * m_tiles * KB
    if p.split_k:
        return Partition(U, KB, p.n_tiles * m_tiles * p.split_k, p.split_k)
    if aligned:
        return Partition(U, KB, p.n_tiles * m_tiles * p.slices, p.slices, lead)
    q = (p.n_tiles * p.m_tiles * KB) // p.grid
    G = max(1, min(p.grid, U // q))
    return Partition(U, KB, G, 0)


def check_tc_partition(p, M_max):
    assert p.tile_n == 128 and p.tile_m in (16, 32, 64, 128, 256) and p.grid >= 1
    assert p.k_step % 64 == 0
    if not p.split_k:
        assert p.grid <= 148 * 2
        assert p.slices == 0 or p.n_tiles * p.m_tiles * p.slices <= 148 * 2
    schedules = [(M, False, 0) for M in sorted({1, M_max, max(1, M_max // 2)})]
    if p.slices:
        # every rank-0 lead the kernel may be built with (nk_common.cuh, NK_TC_LEAD_*)
        schedules += [(M, True, lead) for M in sorted({1, M_max}) for lead in range(0, 9)]
    for M, aligned, lead in schedules:
        P = launch_partition(p, M, aligned, lead)
        assert P.begin(0) == 0 and P.begin(P.G) == P.U
        cover = []
        for c in range(P.G):
            b, e = P.begin(c), P.begin(c + 1)
            assert e > b, "empty CTA range"
            assert P.cta_of(b) == c and P.cta_of(e - 1) == c
            cover.append(e - b)
        assert sum(cover) == P.U
        assert max(cover) - min(cover) <= (1 if not P.split else P.KB)
        T = P.U // P.KB
        for t in range(T):
            nseg = P.cta_of((t + 1) * P.KB - 1) - P.cta_of(t * P.KB) + 1
            assert 1 <= nseg <= p.segments, (t, nseg, p.segments)
        # The finishing protocol of nk_tc.cu relies on: in every CTA's range, a partial
        # segment of rank 0 (it holds the tile's first K block) can only be the CTA's last
        # segment, and one of rank >= 1 only its first; so a waiting rank-0 CTA only waits for
        # higher CTAs that publish before they could wait themselves.
        for c in range(P.G):
            b, e = P.begin(c), P.begin(c + 1)
            u, segs = b, []
            while u < e:
                t = u // P.KB
                end = min(e, (t + 1) * P.KB)
                whole = (u == t * P.KB and end == (t + 1) * P.KB)
                rank = c - P.cta_of(t * P.KB)
                segs.append((whole, rank))
                u = end
            for i, (whole, rank) in enumerate(segs):
                if whole:
                    assert rank == 0
                elif rank == 0:
                    assert i == len(segs) - 1, (c, segs)
                else:
                    assert i == 0, (c, segs)


@pytest.mark.parametrize("N,K", [(6144, 4096), (4096, 4096), (24576, 4096), (4096, 12288),
                                 (151936, 4096), (1024, 2048), (777, 520), (130, 64), (8, 8)])
@pytest.mark.parametrize("M", (1, 4, 16, 17, 64, 100, 256, 300))
@pytest.mark.parametrize("split", (0, 1, 2, 7, 16))
def test_tc_partition_covers_units_once(M, N, K, split):
    st, p = make(M, N, K, split, _lib.KIND_TC)
    assert st == 0 and p.kind == _lib.KIND_TC
    check_tc_partition(p, M)
    ws = _lib.load().nk_ws_bytes(ctypes.byref(p))
    if p.segments > 1:
        cols = min(M, p.tile_m)
        assert ws >= 262144 + p.n_tiles * p.m_tiles * p.segments * cols * 128 * 4
    else:
        assert ws == 0


@pytest.mark.parametrize("M,N,K,slices", [
    (1, 4096, 4096, 9), (8, 4096, 4096, 9), (16, 4096, 4096, 7),   # Qwen3-8B o_proj
    (1, 6144, 4096, 6), (16, 6144, 4096, 6),                         # QKV
    (1, 4096, 12288, 9), (16, 4096, 12288, 7),                       # down
    (1, 24576, 4096, 0), (16, 151936, 4096, 0),                      # gate_up, lm_head
    (64, 4096, 4096, 0), (256, 4096, 4096, 0),                       # verify tiles: one CTA per SM
    (1, 1024, 2048, 8), (16, 1024, 3072, 7), (4, 4096, 1024, 4),     # Qwen3-0.6B
    (1, 8, 256, 0), (32, 6144, 4096, 0)])                            # two K steps; 32-token tile
def test_tile_aligned_slices(M, N, K, slices):
    """The planner's tile-aligned schedule: slices = min(296 // tiles, 9 (7 above M = 8),
    K steps // 2) when that is at least 4, for the 16-token tile (two CTAs per SM)."""
    st, p = make(M, N, K, 0, _lib.KIND_TC)
    assert st == 0 and p.split_k == 0
    assert p.slices == slices, p.as_dict()
    assert p.segments >= slices


def test_generic_plan_for_unaligned_K():
    st, p = make(5, 100, 1001)
    assert st == 0 and p.kind == _lib.KIND_GENERIC and p.split_k == 1


def call(plan, x=0x10000, ldx=None, w=0x20000, ldw=None, y=0x30000, ldy=None, M=1, N=None,
         K=None, ws=None, ws_bytes=0):
    L = _lib.load()
    N = plan.N if N is None else N
    K = plan.K if K is None else K
    return L.nk_gemm_bf16(x, ldx or K, w, ldw or K, y, ldy or N, M, N, K,
                          ctypes.byref(plan) if plan is not None else None, ws, ws_bytes, None)


def test_gemm_rejects_before_launch():
    st, p = make(4, 4096, 1024, 1)
    assert st == 0
    assert call(None, N=4096, K=1024) == _lib.NK_ERR_PLAN
    assert call(p, N=4095) == _lib.NK_ERR_PLAN
    assert call(p, K=2048) == _lib.NK_ERR_PLAN
    assert call(p, M=5) == _lib.NK_ERR_SHAPE
    assert call(p, M=0) == _lib.NK_ERR_SHAPE
    assert call(p, x=0) == _lib.NK_ERR_ARG
    assert call(p, ldx=1000) == _lib.NK_ERR_SHAPE
    assert call(p, x=0x10008) == _lib.NK_ERR_ALIGN       # GEMV needs 16-byte rows
    assert call(p, ldw=1028) == _lib.NK_ERR_ALIGN
    assert call(p, y=0x30001) == _lib.NK_ERR_ALIGN
    st, p4 = make(4, 4096, 1024, 4)
    assert p4.split_k == 4
    assert call(p4) == _lib.NK_ERR_WORKSPACE
    need = _lib.load().nk_ws_bytes(ctypes.byref(p4))
    assert call(p4, ws=0x40000, ws_bytes=need - 1) == _lib.NK_ERR_WORKSPACE
    assert call(p4, ws=0x40010, ws_bytes=need) == _lib.NK_ERR_ALIGN
    corrupt = _lib.NkPlan.from_buffer_copy(p)
    corrupt.magic = 0
    assert call(corrupt) == _lib.NK_ERR_PLAN


def test_python_shim_rejects_cpu_tensors():
    import torch
    a = torch.zeros(2, 8, dtype=torch.bfloat16)
    w = torch.zeros(4, 8, dtype=torch.bfloat16)
    out = torch.empty(2, 4, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        nk.mm(a, w.t(), out=out)
    with pytest.raises(ValueError, match="bfloat16"):
        nk.mm(a.float(), w.t(), out=out)


def test_m_bucket():
    assert [nk.m_bucket(m) for m in (1, 2, 3, 4, 5, 8, 9, 16, 17, 64, 100, 256)] == \
        [1, 2, 4, 4, 8, 8, 16, 16, 32, 64, 112, 256]


def test_argmax_entry_rejects_before_launch():
    L = _lib.load()
    st, p = make(16, 151936, 4096)
    assert st == 0 and p.kind == _lib.KIND_TC
    need = L.nk_gemm_argmax_ws_bytes(ctypes.byref(p))
    assert need >= 288 * 1024 and need >= L.nk_ws_bytes(ctypes.byref(p)) and need % 256 == 0
    st, g = make(4, 4096, 1024, 0, _lib.KIND_GEMV)
    assert st == 0 and L.nk_gemm_argmax_ws_bytes(ctypes.byref(g)) == 0
    st, big = make(1024, 4096, 4096)
    assert st == 0 and L.nk_gemm_argmax_ws_bytes(ctypes.byref(big)) == 0  # > 255 tokens

    def am(plan, y=0x30000, idx=0x50000, best=None, M=1, ws=0x100000, ws_bytes=need):
        return L.nk_gemm_bf16_argmax(0x10000, plan.K, 0x20000, plan.K, y, plan.N, idx, best,
                                     M, plan.N, plan.K, ctypes.byref(plan), ws, ws_bytes, None)

    assert am(g) == _lib.NK_ERR_PLAN
    assert am(big, M=1) == _lib.NK_ERR_SHAPE
    assert am(p, idx=None) == _lib.NK_ERR_ARG
    assert am(p, idx=0x50004) == _lib.NK_ERR_ALIGN
    assert am(p, best=0x60001) == _lib.NK_ERR_ALIGN
    assert am(p, ws=None) == _lib.NK_ERR_WORKSPACE
    assert am(p, ws_bytes=need - 1) == _lib.NK_ERR_WORKSPACE
    assert am(p, ws=0x100010) == _lib.NK_ERR_ALIGN
    assert am(p, M=17) == _lib.NK_ERR_SHAPE
    # no logits: y may be NULL, but nk_gemm_bf16 itself still needs y
    assert am(p, y=None, ws=0x100010) == _lib.NK_ERR_ALIGN
    assert call(p, y=0) == _lib.NK_ERR_ARG


def test_python_greedy_head_rejects_bad_arguments():
    import torch
    a = torch.zeros(2, 8, dtype=torch.bfloat16)
    w = torch.zeros(4, 8, dtype=torch.bfloat16)
    idx = torch.empty(2, dtype=torch.int64)
    with pytest.raises(ValueError, match="CUDA"):
        nk.mm_argmax(a, w.t(), idx=idx)
    with pytest.raises(ValueError, match="bfloat16"):
        nk.mm_argmax(a.float(), w.t(), idx=idx)


def _amax_key(h, n):
    """The greedy head's key (nk_tc.cu amax_key) for bf16 bits h at vocabulary index n."""
    h = 0 if h == 0x8000 else h
    if (h & 0x7FFF) > 0x7F80:
        o = 0xFFFF
    elif h & 0x8000:
        o = ~h & 0xFFFF
    else:
        o = h | 0x8000
    return (o << 32) | (0xFFFFFFFF - n)


def test_greedy_head_key_order_is_torch_argmax_order():
    """The largest key is torch.argmax's choice over the same bf16 row: the largest value, the
    lowest index among equal values, -0 equal to +0, a NaN above everything (first NaN)."""
    import torch
    g = torch.Generator().manual_seed(5)
    specials = torch.tensor([0.0, -0.0, float("inf"), -float("inf"), 1e-40, -1e-40, 3.0, -3.0],
                            dtype=torch.bfloat16)
    for trial in range(300):
        n = int(torch.randint(1, 64, (1,), generator=g))
        row = (torch.randn(n, generator=g) * 4).round().to(torch.bfloat16)  # many ties
        if trial % 3 == 0:
            k = int(torch.randint(0, n, (1,), generator=g))
            row[k] = specials[trial % len(specials)]
        if trial % 50 == 7:
            row[n // 2] = float("nan")
        bits = row.view(torch.int16).to(torch.int32) & 0xFFFF
        keys = [_amax_key(int(b), i) for i, b in enumerate(bits)]
        best = max(range(n), key=lambda i: keys[i])
        assert best == int(torch.argmax(row.float())), (trial, row.tolist())


def test_static_entry_rejects_before_touching_its_scratch():
    """nk_gemm_bf16_static checks every argument before it clears or uses the library's
    scratch array, so a refused call reaches neither the device nor the array."""
    L = _lib.load()
    f = L.nk_gemm_bf16_static
    vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    f.argtypes = [vp, i64, vp, i64, vp, i64, i32, i32, i32, ctypes.POINTER(_lib.NkPlan), vp]
    f.restype = i32
    st, p = make(4, 4096, 4096, 0, _lib.KIND_TC)
    assert st == 0 and L.nk_ws_bytes(ctypes.byref(p)) > 0

    def sc(plan=p, x=0x10000, ldx=4096, w=0x20000, ldw=4096, y=0x30000, ldy=4096, M=4):
        return f(x, ldx, w, ldw, y, ldy, M, 4096, 4096,
                 ctypes.byref(plan) if plan is not None else None, None)

    assert sc(plan=None) == _lib.NK_ERR_PLAN
    assert sc(M=5) == _lib.NK_ERR_SHAPE
    assert sc(x=0) == _lib.NK_ERR_ARG
    assert sc(x=0x10008) == _lib.NK_ERR_ALIGN
    assert sc(ldw=4100) == _lib.NK_ERR_ALIGN
    assert sc(y=0x30001) == _lib.NK_ERR_ALIGN
    assert sc(ldy=100) == _lib.NK_ERR_SHAPE
    # with valid arguments the next check is the device (there is none here)
    assert sc() in (_lib.NK_ERR_CUDA, _lib.NK_ERR_DEVICE)


def test_withhold_request_rejects_bad_tile():
    L = _lib.load()
    assert L.nk_test_withhold_partial(-5) == _lib.NK_ERR_ARG
    assert L.nk_test_withhold_partial(-1) == 0
