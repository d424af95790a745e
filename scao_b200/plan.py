"""Static execution plan: parameter/leaf/tile tables and device arenas.

Built once on the first ``SCAO.step`` (scao/optimizer.py:407-433 initialises
per-parameter state lazily in the same place).  Every Kronecker leaf block of
the reference's recursive block-diagonal split (scao/preconditioner.py:142-194)
becomes one row of the leaf table; moment buffers live in flat fp32 arenas so
one kernel launch per phase covers every parameter.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _lib
from ._lib import CHUNK_DT, LEAF_DT, PANEL_DT, PARAM_DT, STEP_DT, STRIP_DT, TILE_DT

TILE = 128       # apply tile edge (apply.cu TC_T)
PANEL = 128      # projection panel rows
CHUNK = 16384    # flat chunk length (elements per block of the flat passes)
SEL = 65536      # elements per chunk of the gradient filter's selection passes
SMAX = 160       # largest eigen subspace width (eig.cu SMAX)

DTYPE_CODE = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16, torch.float16: _lib.F16}


def to_2d_shape(shape):
    """utils.py:208-219."""
    if len(shape) == 1:
        return 1, shape[0]
    if len(shape) == 2:
        return shape[0], shape[1]
    n = 1
    for d in shape[1:]:
        n *= d
    return shape[0], n


def split_blocks(m, n, mpd):
    """Blocks (row0, col0, a, b) of the recursive block-diagonal split of
    preconditioner.py:142-194.  A block of width 1 (a == 1 or b == 1, the
    remainder of a dimension one above a multiple of max_precond_dim) is a
    diagonal sub-preconditioner there (:142-156, 232-236): it is returned as
    is and becomes a diagonal strip of the plan."""
    if max(m, n) <= mpd:
        return [(0, 0, m, n)]
    large, small = (m, n) if m >= n else (n, m)
    sizes = [mpd] * (large // mpd) + ([large % mpd] if large % mpd else [])
    out, off = [], 0
    for bs in sizes:
        bm, bn = (bs, small) if m >= n else (small, bs)
        sub = [(0, 0, bm, bn)] if bm <= 1 or bn <= 1 else split_blocks(bm, bn, mpd)
        for (r, c, a, b) in sub:
            out.append((r + off, c, a, b) if m >= n else (r, c + off, a, b))
        off += bs
    return out


def split_tree(m, n, mpd):
    """Nesting of the block split: 1 for a Kronecker block, 0 for a diagonal
    (width-1) block, or a list of sub-trees for a block-diagonal one (the
    reference's ``_blocks`` hierarchy, preconditioner.py:163-194)."""
    if m <= 1 or n <= 1:
        return 0
    if max(m, n) <= mpd:
        return 1
    large, small = (m, n) if m >= n else (n, m)
    sizes = [mpd] * (large // mpd) + ([large % mpd] if large % mpd else [])
    return [split_tree(*((bs, small) if m >= n else (small, bs)), mpd) for bs in sizes]


def _round_up(x, k):
    return (x + k - 1) // k * k


def k_bounds(m, n, k_min, k_max):
    """preconditioner.py:122-124."""
    d_min = min(m, n)
    kmin = min(k_min, d_min)
    kmax = min(k_max, d_min // 2) if d_min > 2 * kmin else kmin
    return kmin, kmax


def subspace_width(n, kpad):
    if n <= SMAX:
        return max(n, kpad)
    return min(n, kpad + max(16, min(32, kpad // 2)))


class Plan:
    """Tables + device arenas for an ordered list of parameters."""

    def __init__(self, params, groups_of, device, int8_ema):
        self.params = params
        self.device = device
        self.int8_ema = bool(int8_ema)
        self.n_params = len(params)
        ptab = np.zeros(self.n_params, PARAM_DT)
        leaves, tiles, panels, chunks, strips = [], [], [], [], []
        self.param_leaves = []
        self.param_strips = []
        self.param_blocks = []     # per param, in split order: ("L", leaf) / ("S", strip)
        self.param_trees = []
        off = 0
        fac_off = 0
        u_off = 0
        h_off = 0
        ev_off = 0
        w_off = 0
        ua_off = ut_off = wa_off = 0
        kpad_max = 0
        self.eps_sparse = []
        self.rho_leaf = []
        for i, p in enumerate(params):
            g = groups_of[i]
            if p.dtype not in DTYPE_CODE:
                raise TypeError(f"unsupported parameter dtype {p.dtype}")
            m, n = to_2d_shape(tuple(p.shape))
            numel = p.numel()
            kron = p.dim() >= 2 and m > 1 and n > 1
            r = ptab[i]
            r["offset"] = off
            r["numel"] = numel
            r["rows"], r["cols"] = m, n
            r["mode"] = 1 if kron else 0
            r["dtype"] = DTYPE_CODE[p.dtype]
            r["leaf_begin"] = len(leaves)
            r["tile_begin"] = len(tiles)
            r["chunk_begin"] = len(chunks)
            mine, mine_s, order = [], [], []
            if kron:
                blocks = split_blocks(m, n, g["max_precond_dim"])
                for (r0, c0, a, b) in blocks:
                    if a == 1 or b == 1:
                        # diagonal strip: a row (stride 1) or a column (stride n)
                        order.append(("S", len(strips)))
                        mine_s.append(len(strips))
                        strips.append((i, b if a == 1 else a, 1 if a == 1 else n, 0,
                                       r0 * n + c0))
                        continue
                    order.append(("L", len(leaves)))
                    kmin, kmax = k_bounds(a, b, g["k_min"], g["k_max"])
                    kpad = _round_up(max(kmax, 1), 8)
                    if kpad > 128:
                        raise NotImplementedError("k_max above 128 is not supported")
                    kpad_max = max(kpad_max, kpad)
                    sl, sr = subspace_width(a, kpad), subspace_width(b, kpad)
                    L = np.zeros((), LEAF_DT)
                    L["param"], L["row0"], L["col0"], L["a"], L["b"] = i, r0, c0, a, b
                    L["ld"] = n
                    L["kmin"], L["kmax"], L["kpad"], L["sl"], L["sr"] = kmin, kmax, kpad, sl, sr
                    L["tile_begin"] = len(tiles)
                    li = len(leaves)
                    for tr in range(0, a, TILE):
                        for tc in range(0, b, TILE):
                            tiles.append((li, tr, tc, 0))
                    L["tile_end"] = len(tiles)
                    L["panel_begin"] = len(panels)
                    for pr in range(0, a, PANEL):
                        panels.append((li, pr, min(PANEL, a - pr), 0))
                    L["panel_end"] = len(panels)
                    L["lq_off"] = fac_off
                    fac_off += _round_up(a * a, 16)
                    L["rq_off"] = fac_off
                    fac_off += _round_up(b * b, 16)
                    L["ul_off"] = u_off
                    u_off += _round_up(a * sl, 4)
                    L["ur_off"] = u_off
                    u_off += _round_up(b * sr, 4)
                    L["hl_off"] = h_off
                    h_off += _round_up(sl * sl, 4)
                    L["hr_off"] = h_off
                    h_off += _round_up(sr * sr, 4)
                    L["evl_off"] = ev_off
                    ev_off += _round_up(sl, 4)
                    L["evr_off"] = ev_off
                    ev_off += _round_up(sr, 4)
                    L["w_off"] = w_off
                    w_off += _round_up(a * kpad, 4)
                    kp16 = _round_up(kpad, 16)
                    L["ua_off"] = ua_off
                    ua_off += -(-b // 128) * 2 * 128 * kp16 * 2
                    L["ut_off"] = ut_off
                    ut_off += -(-b // 64) * 2 * kp16 * 64 * 2
                    L["wa_off"] = wa_off
                    wa_off += -(-a // 128) * 2 * 128 * kp16 * 2
                    leaves.append(L)
                    mine.append(li)
                    self.eps_sparse.append(g["epsilon_sparse"])
                    self.rho_leaf.append(g["rho"])
            if kron and not mine:
                raise NotImplementedError(
                    f"max_precond_dim={g['max_precond_dim']} leaves no Kronecker block in a "
                    f"{m}x{n} parameter")
            self.param_leaves.append(mine)
            self.param_strips.append(mine_s)
            self.param_blocks.append(order)
            self.param_trees.append(split_tree(m, n, g["max_precond_dim"]) if kron else 0)
            r["leaf_end"] = len(leaves)
            r["tile_end"] = len(tiles)
            for c0 in range(0, numel, CHUNK):
                chunks.append((i, 0, c0, min(numel, c0 + CHUNK)))
            r["chunk_end"] = len(chunks)
            off += _round_up(numel, 8)     # 16-byte aligned in the bf16 arenas too
        self.numel_total = off
        self.ptab = ptab
        self.ltab = np.array(leaves, LEAF_DT) if leaves else np.zeros(0, LEAF_DT)
        self.ttab = np.array(tiles, TILE_DT) if tiles else np.zeros(0, TILE_DT)
        self.pantab = np.array(panels, PANEL_DT) if panels else np.zeros(0, PANEL_DT)
        self.ctab = np.array(chunks, CHUNK_DT) if chunks else np.zeros(0, CHUNK_DT)
        self.stab = np.array(strips, STRIP_DT) if strips else np.zeros(0, STRIP_DT)
        self.n_strips = len(strips)
        self.kpad_max = kpad_max
        self.p_stride = kpad_max * kpad_max + 4
        self.n_leaves = len(leaves)
        self._tile_bytes = (ua_off, ut_off, wa_off)
        self._alloc(fac_off, u_off, h_off, ev_off, w_off)

    # ------------------------------------------------------------------
    def _dev(self, arr):
        t = torch.from_numpy(np.ascontiguousarray(arr).view(np.uint8).copy())
        return t.to(self.device)

    def _alloc(self, fac_n, u_n, h_n, ev_n, w_n):
        dev = self.device
        z = lambda n, dt=torch.float32: torch.zeros(max(int(n), 1), dtype=dt, device=dev)
        self.t_params = self._dev(self.ptab)
        self.t_leaves = self._dev(self.ltab) if self.n_leaves else z(1)
        self.t_tiles = self._dev(self.ttab) if len(self.ttab) else z(1)
        self.t_panels = self._dev(self.pantab) if len(self.pantab) else z(1)
        self.t_chunks = self._dev(self.ctab) if len(self.ctab) else z(1)
        self.t_strips = self._dev(self.stab) if self.n_strips else z(1)
        self.strip_part = z(self.n_strips * 4)
        self.step_host = torch.zeros(self.n_params * STEP_DT.itemsize, dtype=torch.uint8,
                                     pin_memory=torch.cuda.is_available())
        self.step_np = self.step_host.numpy().view(STEP_DT)
        self.step_event = None
        self.t_step = torch.zeros(self.n_params * STEP_DT.itemsize, dtype=torch.uint8,
                                  device=dev)
        N = self.numel_total
        self.exp_avg, self.exp_avg_sq = z(N), z(N)
        self.exp_avg_diff, self.prev_grad = z(N), z(N)
        self.diag_ema = z(N)
        if self.int8_ema:
            self.fac = z(fac_n, torch.int8)
        else:
            self.fac = z(fac_n)
        self.absmax = z(2 * self.n_leaves)
        self.u = z(u_n)
        self.ev = z(ev_n)
        self.k = z(self.n_leaves, torch.int32)
        self.eig_y, self.eig_x, self.eig_ax = z(u_n), z(u_n), z(u_n)
        self.eig_h, self.eig_v = z(h_n), z(h_n)
        # split-bf16 images of the eigensolver's n x s operands (subspace
        # problems): 64-row chunks x 16-padded width x 3 bf16 parts
        stride = 16
        for li in range(self.n_leaves):
            for side in (0, 1):
                n = int(self.ltab["b" if side else "a"][li])
                sw = int(self.ltab["sr" if side else "sl"][li])
                if sw < n:
                    stride = max(stride, _round_up(n, 64) * _round_up(sw, 16) * 6)
        self.eig_img_stride = stride
        self.eig_img = z(stride * 2 * self.n_leaves if stride > 16 else 16, torch.uint8)
        self.eig_aux = z(2 * self.n_leaves * 16)
        self.eig_status = z(2 * self.n_leaves, torch.int32)
        self.w = z(w_n)
        self.p_part = z(len(self.pantab) * self.p_stride)
        self.tile_part = z(len(self.ttab) * 4)
        self.chunk_part = z(len(self.ctab) * 4)
        has16 = any(p.dtype != torch.float32 for p in self.params)
        has32 = any(p.dtype == torch.float32 for p in self.params)
        self.upd = z(N if has16 else 1, torch.int16)
        self.upd32 = z(N if has32 else 1)
        self.leaf_nat2 = z(self.n_leaves)
        self.param_scalars = z(self.n_params * 8)
        self.global_norm_ema = torch.ones(1, dtype=torch.float64, device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        self.err_pin = torch.zeros(1, dtype=torch.int32, pin_memory=torch.cuda.is_available())
        self.err_event = None
        self.tmaps = torch.zeros(self.n_params * 10 * 128, dtype=torch.uint8, device=dev)
        self.tmap_cache = {}          # pointer-set key -> device buffer of maps (LRU order)
        # leaves whose panels the TMA projection can take (static part of its
        # test: bf16, 16-byte aligned rows and block origin, 64-multiple width)
        self.leaf_tma_shape = np.array(
            [int(self.ptab[int(L["param"])]["dtype"]) == DTYPE_CODE[torch.bfloat16] and
             int(L["ld"]) % 8 == 0 and int(L["col0"]) % 8 == 0 and int(L["b"]) % 64 == 0
             for L in self.ltab], dtype=bool) if self.n_leaves else np.zeros(0, bool)
        self.leaf_param = self.ltab["param"].astype(np.int64) if self.n_leaves else np.zeros(0, np.int64)
        # ... and whose tiles the TMA apply can take (whole 128 x 128 tiles)
        self.leaf_tma_apply = np.array(
            [int(self.ptab[int(L["param"])]["dtype"]) == DTYPE_CODE[torch.bfloat16] and
             int(L["ld"]) % 8 == 0 and int(L["col0"]) % 8 == 0 and int(L["a"]) % 128 == 0 and
             int(L["b"]) % 128 == 0 and int(self.ptab[int(L["param"])]["offset"]) % 8 == 0
             for L in self.ltab], dtype=bool) if self.n_leaves else np.zeros(0, bool)
        self.has_bf16_kron = any(int(r["mode"]) == 1 and int(r["dtype"]) == DTYPE_CODE[torch.bfloat16]
                                 for r in self.ptab)
        self.counters = z(16, torch.int32)
        nc = max(len(self.ctab), 1)
        self.t_diag_list = z(nc, torch.int32)
        self.t_flat_list = z(nc, torch.int32)
        self.t_p_list = z(nc, torch.int32)
        self._chunk_param = self.ctab["param"].astype(np.int64) if len(self.ctab) else np.zeros(0, np.int64)
        diag = np.nonzero(self.ptab["mode"][self._chunk_param] == 0)[0].astype(np.int32) \
            if len(self.ctab) else np.zeros(0, np.int32)
        if len(diag):
            self.t_diag_list[:len(diag)].copy_(torch.from_numpy(diag))
        self.n_diag = len(diag)
        self._phase_key = None
        self.ua = z(self._tile_bytes[0], torch.uint8)
        self.ut = z(self._tile_bytes[1], torch.uint8)
        self.wa = z(self._tile_bytes[2], torch.uint8)
        self.slow = None
        self.slow32 = None
        self.t_eps_sparse = torch.tensor(self.eps_sparse or [0.0], dtype=torch.float32,
                                         device=dev)
        self.t_bias = torch.zeros(max(self.n_leaves, 1), dtype=torch.float32, device=dev)
        self.t_bias_host = np.zeros(self.n_leaves, np.float32)
        self._ids_cache = {}
        self._init_factors()
        self.dev = PlanDev_from(self)
        if self.n_leaves and self.device.type == "cuda":
            import ctypes
            ids = torch.arange(self.n_leaves, dtype=torch.int32, device=dev)
            _lib.check(_lib.lib().scao_plan_prep_factors(
                ctypes.byref(self.dev), ids.data_ptr(), self.n_leaves,
                torch.cuda.current_stream(dev).cuda_stream), "scao_plan_prep_factors")

    def prep_leaves(self, leaf_ids):
        """Rebuild the eigenvector operand tiles of the listed leaves (after
        their U / S were written from the host, e.g. by a checkpoint load)."""
        if not len(leaf_ids) or self.device.type != "cuda":
            return
        import ctypes
        ids = torch.tensor(list(leaf_ids), dtype=torch.int32, device=self.device)
        _lib.check(_lib.lib().scao_plan_prep_factors(
            ctypes.byref(self.dev), ids.data_ptr(), len(leaf_ids),
            torch.cuda.current_stream(self.device).cuda_stream), "scao_plan_prep_factors")
        torch.cuda.current_stream(self.device).synchronize()

    def _init_factors(self):
        """L = R = 1e-4*I (int8: q = 127*I, absmax = float32(1e-4)), U = reversed
        identity (warm start; unused until the first eigen update), S = 1 for
        the first k_init columns (preconditioner.py:196-231)."""
        if not self.n_leaves:
            return
        L = self.ltab
        fac = torch.zeros_like(self.fac, device="cpu")
        u = torch.zeros(self.u.numel(), dtype=torch.float32)
        ev = torch.zeros(self.ev.numel(), dtype=torch.float32)
        eye_val = np.float32(1e-4)
        for li in range(self.n_leaves):
            for side in (0, 1):
                n = int(L["a"][li] if side == 0 else L["b"][li])
                s = int(L["sl"][li] if side == 0 else L["sr"][li])
                fo = int(L["lq_off"][li] if side == 0 else L["rq_off"][li])
                uo = int(L["ul_off"][li] if side == 0 else L["ur_off"][li])
                eo = int(L["evl_off"][li] if side == 0 else L["evr_off"][li])
                d = torch.arange(n)
                if self.int8_ema:
                    fac[fo + d * n + d] = 127
                else:
                    fac[fo + d * n + d] = float(eye_val)
                c = torch.arange(min(n, s))
                u[uo + (n - 1 - c) * s + c] = 1.0
                ev[eo: eo + int(L["kmin"][li])] = 1.0
        self.fac.copy_(fac)
        self.u.copy_(u)
        self.ev.copy_(ev)
        self.absmax.fill_(float(eye_val))
        self.k.copy_(torch.from_numpy(L["kmin"].astype(np.int32)))

    def set_phases(self, phases):
        """Chunk lists for the flat passes of this step (re-uploaded only when
        the per-parameter phase vector changes)."""
        key = phases.tobytes()
        if key == self._phase_key:
            return
        self._phase_key = key
        if len(self.ctab):
            ph = phases[self._chunk_param]
            mode = self.ptab["mode"][self._chunk_param]
            flat = np.nonzero((ph == 1) | ((ph == 2) & (mode == 0)))[0].astype(np.int32)
            pl = np.nonzero(ph == 2)[0].astype(np.int32)
        else:
            flat = pl = np.zeros(0, np.int32)
        if len(flat):
            self.t_flat_list[:len(flat)].copy_(torch.from_numpy(flat))
        if len(pl):
            self.t_p_list[:len(pl)].copy_(torch.from_numpy(pl))
        self.dev.n_flat = len(flat)
        self.dev.n_p = len(pl)

    def setup_filter(self, mode, sparsity, ema=0.99):
        """Device state of the sparse gradient filter (optimizer.py:40-97):
        magnitude-EMA arena, selection chunks of <= SEL elements per param,
        per-param radix-selection state.  ``mode`` 1 static, 2 dynamic (R2)."""
        f = self.dev.filt
        if f.mode:
            return
        sel = []
        fp = np.zeros(self.n_params, _lib.FILTER_PARAM_DT)
        for i in range(self.n_params):
            n = int(self.ptab[i]["numel"])
            fp[i]["sel_begin"] = len(sel)
            for c0 in range(0, n, SEL):
                sel.append((i, 0, c0, min(n, c0 + SEL)))
            fp[i]["sel_end"] = len(sel)
        fp["norm_ema"] = 1.0
        fp["global_ref"] = 1.0
        fp["first"] = 1
        dev = self.device
        self.t_sel = self._dev(np.array(sel, CHUNK_DT))
        self.t_fp = self._dev(fp)
        self.mag_ema = torch.zeros(max(self.numel_total, 1), dtype=torch.float32, device=dev)
        self.filt_hist = torch.zeros(self.n_params * 2 * 4096, dtype=torch.int32, device=dev)
        self.sel_part = torch.zeros(max(len(sel), 1), dtype=torch.float32, device=dev)
        f.mode = int(mode)
        f.n_sel = len(sel)
        f.sel, f.mag_ema, f.fp = self.t_sel.data_ptr(), self.mag_ema.data_ptr(), self.t_fp.data_ptr()
        f.hist, f.sel_part = self.filt_hist.data_ptr(), self.sel_part.data_ptr()
        f.base, f.min_s, f.max_s, f.norm_coeff = float(sparsity), 0.3, 0.9, 0.95
        f.ema = float(np.float32(ema))
        f.ema_c = float(np.float32(1.0 - ema))

    def filter_params(self):
        """Per-parameter filter state (numpy copy; synchronises)."""
        if not self.dev.filt.mode:
            return None
        return self.t_fp.cpu().numpy().view(_lib.FILTER_PARAM_DT)

    # host -> device uploads without a stream synchronisation -------------
    def dev_ids(self, ids_h):
        """Device copy of an int32 id list, cached by content (the lists a
        step uses repeat with the curvature cadence)."""
        key = ids_h.tobytes()
        t = self._ids_cache.get(key)
        if t is None:
            t = torch.from_numpy(ids_h.copy()).to(self.device)
            self._ids_cache[key] = t
        return t

    def _pinned(self, name, n, dtype):
        buf = getattr(self, name, None)
        ev = getattr(self, name + "_ev", None)
        if ev is not None:
            ev.synchronize()            # the previous upload has left the buffer
        if buf is None or buf.numel() < n:
            buf = torch.zeros(max(n, 1), dtype=dtype, pin_memory=torch.cuda.is_available())
            setattr(self, name, buf)
        return buf

    def _mark(self, name):
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        setattr(self, name + "_ev", ev)

    def upload_bias(self, leaf_ids, values):
        """t_bias[leaf_ids] = values, from pinned memory, stream-ordered."""
        buf = self._pinned("_bias_pin", self.n_leaves, torch.float32)
        arr = buf.numpy()
        arr[:self.n_leaves] = self.t_bias_host
        arr[leaf_ids] = np.asarray(values, np.float32)
        self.t_bias_host[:] = arr[:self.n_leaves]
        self.t_bias[:self.n_leaves].copy_(buf[:self.n_leaves], non_blocking=True)
        self._mark("_bias_pin")
        return self.t_bias

    def upload_k(self, kvec):
        buf = self._pinned("_k_pin_up", self.n_leaves, torch.int32)
        buf.numpy()[:self.n_leaves] = kvec
        self.k.copy_(buf[:self.n_leaves], non_blocking=True)
        self._mark("_k_pin_up")

    def select_tensor_maps(self, key, pd, stream, keep=4):
        """Point the plan at the tensor maps of ``key`` (gradient / parameter
        pointers and phases), encoding them on a miss.  Buffers are reused in
        LRU order; a rewrite is stream-ordered after the kernels that read it."""
        buf = self.tmap_cache.pop(key, None)
        hit = buf is not None
        if not hit:
            if len(self.tmap_cache) >= keep:
                old = next(iter(self.tmap_cache))
                buf = self.tmap_cache.pop(old)
            else:
                buf = torch.zeros(self.n_params * 10 * 128, dtype=torch.uint8, device=self.device)
        self.tmap_cache[key] = buf
        self.tmaps = buf
        self.dev.tmaps = buf.data_ptr()
        if hit:
            self.dev.tmaps_ok = 1
            return
        rc = _lib.lib().scao_plan_tensor_maps(pd, self.ptab.ctypes.data, self.step_host.data_ptr(),
                                              stream)
        self.dev.tmaps_ok = 1 if rc == 0 else 0
        if rc != 0:
            self.tmap_cache.pop(key, None)

    def check_error(self):
        """Raise if a kernel recorded a timed-out wait (synchronises)."""
        if int(self.err.item()):
            raise RuntimeError("scao_b200: a tensor-core completion wait timed out")

    def ensure_slow(self):
        if self.slow is None:
            N = self.numel_total
            self.slow = torch.zeros(N, dtype=torch.int16, device=self.device)
            self.slow32 = torch.zeros(N, dtype=torch.float32, device=self.device)
            self.dev.slow = self.slow.data_ptr()
            self.dev.slow32 = self.slow32.data_ptr()

    # views ------------------------------------------------------------
    def state_view(self, arena, i):
        r = self.ptab[i]
        o, n = int(r["offset"]), int(r["numel"])
        return arena[o:o + n].view(self.params[i].shape)

    def max_dims(self, leaf_ids):
        L = self.ltab[leaf_ids]
        return int(L["a"].max()), int(L["b"].max()), int(max(L["sl"].max(), L["sr"].max()))


def PlanDev_from(plan):
    d = _lib.PlanDev()
    d.n_params = plan.n_params
    d.n_leaves = plan.n_leaves
    d.n_tiles = len(plan.ttab)
    d.n_panels = len(plan.pantab)
    d.n_chunks = len(plan.ctab)
    d.int8_ema = int(plan.int8_ema)
    d.kpad_max = plan.kpad_max
    d.p_stride = plan.p_stride
    d.max_leaf_rows_tiles = int((-(-plan.ltab["a"] // 128)).max()) if plan.n_leaves else 0
    d.kron_dtypes = int(np.bitwise_or.reduce(
        [1 << int(r["dtype"]) for r in plan.ptab if int(r["mode"]) == 1] or [0]))
    ptr = lambda t: t.data_ptr() if t is not None else None
    d.params, d.leaves, d.tiles = ptr(plan.t_params), ptr(plan.t_leaves), ptr(plan.t_tiles)
    d.panels, d.chunks, d.step = ptr(plan.t_panels), ptr(plan.t_chunks), ptr(plan.t_step)
    d.exp_avg, d.exp_avg_sq = ptr(plan.exp_avg), ptr(plan.exp_avg_sq)
    d.exp_avg_diff, d.prev_grad = ptr(plan.exp_avg_diff), ptr(plan.prev_grad)
    d.diag_ema, d.fac, d.absmax = ptr(plan.diag_ema), ptr(plan.fac), ptr(plan.absmax)
    d.u, d.ev, d.k = ptr(plan.u), ptr(plan.ev), ptr(plan.k)
    d.eig_y, d.eig_x, d.eig_ax = ptr(plan.eig_y), ptr(plan.eig_x), ptr(plan.eig_ax)
    d.eig_h, d.eig_v, d.eig_aux = ptr(plan.eig_h), ptr(plan.eig_v), ptr(plan.eig_aux)
    d.w, d.p_part, d.tile_part = ptr(plan.w), ptr(plan.p_part), ptr(plan.tile_part)
    d.chunk_part, d.upd, d.upd32 = ptr(plan.chunk_part), ptr(plan.upd), ptr(plan.upd32)
    d.leaf_nat2, d.param_scalars = ptr(plan.leaf_nat2), ptr(plan.param_scalars)
    d.global_norm_ema = ptr(plan.global_norm_ema)
    d.err = ptr(plan.err)
    d.tmaps = ptr(plan.tmaps)
    d.ua, d.ut, d.wa = ptr(plan.ua), ptr(plan.ut), ptr(plan.wa)
    d.counters = ptr(plan.counters)
    d.diag_list, d.flat_list, d.p_list = ptr(plan.t_diag_list), ptr(plan.t_flat_list), ptr(plan.t_p_list)
    d.n_diag = plan.n_diag
    d.strips, d.strip_part, d.n_strips = ptr(plan.t_strips), ptr(plan.strip_part), plan.n_strips
    d.eig_img = ptr(plan.eig_img)
    d.eig_img_stride = plan.eig_img_stride
    return d
