"""Host-side mirror of the slam-hands correlation interface over libdroidcorr.

`DroidCorrelation` keeps the names, argument meanings and buffer layouts of the
correlation methods of `CudaDroid` (cuda_slam/main.cu:1499-1613; the same
methods at cuda_pipeline/slam.cuh:2796-2909):

  build_correlation(i, j)                          main.cu:1500
  sample_correlation(coords_2hw, corr_out)         main.cu:1529
  batch_build_and_sample_correlation(batch_size, edge_start, coords_2hw,
                                     corr_out_196hw)  main.cu:1555

plus tensor-level calls (build_volume, lookup, build_and_lookup, alt_lookup).
Device memory comes from PyTorch tensors (plumbing only); every computation is
a call into the CUDA library.  Errors raise DroidCorrError with the library's
message (the reference exits the process instead, cuda_slam/nn.cuh:17-41).
"""
from __future__ import annotations

import ctypes
from typing import List, Optional, Sequence

import torch

from . import _lib as L


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(stream: Optional[torch.cuda.Stream]) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


class DroidCorrelation:
    """One correlation context on one GPU (the correlation state of CudaDroid)."""

    def __init__(self, h: int, w: int, channels: int = 128, levels: int = 4, radius: int = 3,
                 max_frames: int = 512, max_edges: int = 48, precision: str = "fp16",
                 alpha: float = 1.0 / 16.0, device: Optional[torch.device] = None):
        self.lib = L.load()
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        if self.device.type != "cuda":
            raise ValueError("DroidCorrelation needs a CUDA device")
        if precision not in L.PRECISIONS:
            raise ValueError(f"precision must be one of {sorted(L.PRECISIONS)}")
        self.h, self.w, self.hw = h, w, h * w
        self.channels, self.levels, self.radius = channels, levels, radius
        self.D = 2 * radius + 1
        self.out_channels = levels * self.D * self.D
        self.max_frames, self.max_edges = max_frames, max_edges
        self.precision, self.alpha = precision, float(alpha)
        cfg = L.DcConfig(h, w, channels, levels, radius, max_frames, max_edges,
                         L.PRECISIONS[precision], float(alpha))
        handle = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            rc = self.lib.dc_create(ctypes.byref(cfg), ctypes.byref(handle))
        if rc != L.DC_OK:
            raise L.DroidCorrError(rc, self.lib.dc_status_string(rc).decode())
        self._ctx = handle
        # edge lists, as DroidState::ii_host / jj_host (main.cu:683)
        self.ii_host: List[int] = []
        self.jj_host: List[int] = []
        # single-edge buffers, as CudaDroid::corr_volume / corr_pyramid (main.cu:1323-1325)
        self.corr_volume: Optional[torch.Tensor] = None
        self.corr_pyramid: List[Optional[torch.Tensor]] = [None] * levels

    # -- lifetime -------------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "_ctx", None):
            self.lib.dc_destroy(self._ctx)
            self._ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc: int) -> None:
        if rc != L.DC_OK:
            msg = self.lib.dc_last_error(self._ctx).decode()
            raise L.DroidCorrError(rc, msg or self.lib.dc_status_string(rc).decode())

    def _cuda(self, t: torch.Tensor, dtype: torch.dtype, name: str) -> torch.Tensor:
        if t.device != self.device or t.dtype != dtype or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous {dtype} tensor on {self.device}")
        return t

    def _edges(self, ii, jj):
        ii = torch.as_tensor(ii, dtype=torch.int32, device=self.device).contiguous()
        jj = torch.as_tensor(jj, dtype=torch.int32, device=self.device).contiguous()
        if ii.shape != jj.shape or ii.dim() != 1:
            raise ValueError("ii and jj must be 1-D of equal length")
        return ii, jj

    @property
    def context_bytes(self) -> int:
        return int(self.lib.dc_context_bytes(self._ctx))

    @property
    def launch_count(self) -> int:
        return int(self.lib.dc_launch_count(self._ctx))

    # -- feature-map store -----------------------------------------------------
    def set_max_ctas(self, max_ctas: int) -> None:
        """Cap the persistent fused kernel's CTAs (0 = one per SM), leaving SMs
        free for work on other streams (dc_set_max_ctas)."""
        self._check(self.lib.dc_set_max_ctas(self._ctx, int(max_ctas)))

    def set_tile_order(self, order: str) -> None:
        """How the fused kernel groups each edge's source pixels into tiles
        (dc_set_tile_order): "source" (consecutive pixels, the default),
        "window_row" (sorted by the row of their level-0 window: fewer target
        rows per tile under large, noisy flow) or "auto" (per edge, the window-row
        order where it saves enough target pixels per tile)."""
        if order not in L.TILE_ORDERS:
            raise ValueError(f"order must be one of {sorted(L.TILE_ORDERS)}")
        self._check(self.lib.dc_set_tile_order(self._ctx, L.TILE_ORDERS[order]))

    def set_frames(self, fmaps: torch.Tensor, first_slot: int = 0,
                   stream: Optional[torch.cuda.Stream] = None) -> None:
        """Pack fmaps [K, C, h, w] (fp32 or fp16) into slots first_slot..+K."""
        if fmaps.dim() != 4 or tuple(fmaps.shape[1:]) != (self.channels, self.h, self.w):
            raise ValueError(f"fmaps must be [K, {self.channels}, {self.h}, {self.w}]")
        if fmaps.dtype == torch.float32:
            dt = L.DC_DTYPE_F32
        elif fmaps.dtype == torch.float16:
            dt = L.DC_DTYPE_F16
        else:
            raise ValueError("fmaps must be float32 or float16")
        self._cuda(fmaps, fmaps.dtype, "fmaps")
        self._check(self.lib.dc_set_frames(self._ctx, fmaps.data_ptr(), dt, first_slot,
                                           fmaps.shape[0], _stream(stream)))

    def store_ipc_handle(self) -> bytes:
        """CUDA IPC handle of the packed store, for dc_store_attach_source in
        another process (dc_store_ipc_handle)."""
        buf = ctypes.create_string_buffer(64)
        self._check(self.lib.dc_store_ipc_handle(self._ctx, buf))
        return buf.raw

    def attach_source(self, handle: bytes) -> None:
        """Open another process's store (same configuration) as the source of
        pull_slots (dc_store_attach_source)."""
        self._check(self.lib.dc_store_attach_source(self._ctx, ctypes.c_char_p(bytes(handle))))

    def pull_slots(self, first_slot: int, count: int,
                   stream: Optional[torch.cuda.Stream] = None) -> None:
        """Copy store slots from the attached source store (copy engine, async)."""
        self._check(self.lib.dc_store_pull_slots(self._ctx, first_slot, count, _stream(stream)))

    def sync_signal(self, word: int, value: int, remote: bool = False,
                    stream: Optional[torch.cuda.Stream] = None) -> None:
        """Stream-ordered write of a replication counter (dc_sync_signal)."""
        self._check(self.lib.dc_sync_signal(self._ctx, word, value, int(remote), _stream(stream)))

    def sync_wait(self, word: int, value: int, remote: bool = False,
                  stream: Optional[torch.cuda.Stream] = None) -> None:
        """Hold the stream until a replication counter reaches value (dc_sync_wait)."""
        self._check(self.lib.dc_sync_wait(self._ctx, word, value, int(remote), _stream(stream)))

    def store_slots(self, first_slot: int, count: int) -> torch.Tensor:
        """uint8 view [bytes] of the packed store slots first_slot..+count (device
        memory owned by the library; valid while this object lives)."""
        ptr, nbytes = ctypes.c_void_p(), ctypes.c_longlong()
        self._check(self.lib.dc_store_slots(self._ctx, first_slot, count, ctypes.byref(ptr),
                                            ctypes.byref(nbytes)))

        class _View:
            __cuda_array_interface__ = {"shape": (nbytes.value,), "typestr": "|u1",
                                        "data": (ptr.value, False), "version": 3}

        return torch.as_tensor(_View(), device=self.device)

    # -- tensor-level calls ----------------------------------------------------
    def volume_shapes(self, M: int):
        return [(M, self.hw, self.h >> l, self.w >> l) for l in range(self.levels)]

    def build_volume(self, ii, jj, vols: Optional[Sequence[torch.Tensor]] = None,
                     stream: Optional[torch.cuda.Stream] = None) -> List[torch.Tensor]:
        """Materialised volume pyramid [M, hw, h>>l, w>>l] for edges (ii, jj)."""
        ii, jj = self._edges(ii, jj)
        M = ii.numel()
        if vols is None:
            vols = [torch.empty(s, dtype=torch.float32, device=self.device)
                    for s in self.volume_shapes(M)]
        for l, v in enumerate(vols):
            if v is not None:
                self._cuda(v, torch.float32, f"vols[{l}]")
        for c0 in range(0, max(M, 1), self.max_edges):
            m = min(self.max_edges, M - c0)
            if m <= 0:
                break
            sub = (ctypes.c_void_p * self.levels)(
                *[None if v is None else v[c0].data_ptr() for v in vols])
            self._check(self.lib.dc_build_volume(self._ctx, ii[c0].data_ptr(),
                                                 jj[c0].data_ptr(), m, sub, _stream(stream)))
        return list(vols)

    def lookup(self, vols: Sequence[torch.Tensor], coords: torch.Tensor,
               out: Optional[torch.Tensor] = None,
               stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        """coords [M, 2, h, w] -> out [M, levels*D*D, h, w] from materialised volumes."""
        self._cuda(coords, torch.float32, "coords")
        M = coords.shape[0]
        if out is None:
            out = torch.empty(M, self.out_channels, self.h, self.w, device=self.device)
        self._cuda(out, torch.float32, "out")
        for l, v in enumerate(vols[: self.levels]):
            self._cuda(v, torch.float32, f"vols[{l}]")
            if v.numel() != M * self.hw * (self.h >> l) * (self.w >> l):
                raise ValueError(f"vols[{l}] has the wrong size")
        arr = (ctypes.c_void_p * self.levels)(*[v.data_ptr() for v in vols[: self.levels]])
        self._check(self.lib.dc_lookup(self._ctx, arr, coords.data_ptr(), out.data_ptr(), M,
                                       _stream(stream)))
        return out

    def lookup_single(self, vols: Sequence[torch.Tensor], coords: torch.Tensor,
                      out: Optional[torch.Tensor] = None,
                      stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        """One edge with the corr_index_kernel arithmetic: coords [2,h,w] -> [196,h,w]."""
        self._cuda(coords, torch.float32, "coords")
        if out is None:
            out = torch.empty(self.out_channels, self.h, self.w, device=self.device)
        self._cuda(out, torch.float32, "out")
        arr = (ctypes.c_void_p * self.levels)(*[v.data_ptr() for v in vols[: self.levels]])
        self._check(self.lib.dc_lookup_single(self._ctx, arr, coords.data_ptr(),
                                              out.data_ptr(), _stream(stream)))
        return out

    def _edge_call(self, fn, ii, jj, coords, out, stream):
        ii, jj = self._edges(ii, jj)
        M = ii.numel()
        self._cuda(coords, torch.float32, "coords")
        if coords.shape != (M, 2, self.h, self.w):
            raise ValueError(f"coords must be [{M}, 2, {self.h}, {self.w}]")
        if out is None:
            out = torch.empty(M, self.out_channels, self.h, self.w, device=self.device)
        self._cuda(out, torch.float32, "out")
        s = _stream(stream)
        for c0 in range(0, M, self.max_edges):
            m = min(self.max_edges, M - c0)
            self._check(fn(self._ctx, ii[c0].data_ptr(), jj[c0].data_ptr(), m,
                           coords[c0].data_ptr(), out[c0].data_ptr(), s))
        return out

    def build_and_lookup(self, ii, jj, coords: torch.Tensor, out: Optional[torch.Tensor] = None,
                         stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        """Fused build + pyramid + lookup (no volume in memory)."""
        return self._edge_call(self.lib.dc_build_and_lookup, ii, jj, coords, out, stream)

    # -- correlation encoder (corr_enc_0 + ReLU + fp16, main.cu:552-553, :603-606) --
    def set_corr_encoder(self, weight: torch.Tensor, bias: torch.Tensor,
                         stream: Optional[torch.cuda.Stream] = None) -> None:
        """weight [128, 196] (or [128, 196, 1, 1]) fp32, bias [128] fp32."""
        w = weight.reshape(weight.shape[0], -1).contiguous()
        if w.shape != (128, self.out_channels):
            raise ValueError(f"weight must be [128, {self.out_channels}]")
        self._cuda(w, torch.float32, "weight")
        self._cuda(bias, torch.float32, "bias")
        self._enc_keep = (w, bias)  # the packing kernel reads them on `stream`
        self._check(self.lib.dc_set_corr_encoder(self._ctx, w.data_ptr(), bias.data_ptr(),
                                                 w.shape[0], _stream(stream)))

    def corr_encode(self, corr: torch.Tensor, out: Optional[torch.Tensor] = None,
                    stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        """fp16(relu(W corr + b)): corr [M, 196, h, w] fp32 -> [M, 128, h, w] fp16."""
        self._cuda(corr, torch.float32, "corr")
        M = corr.shape[0]
        if corr.shape != (M, self.out_channels, self.h, self.w):
            raise ValueError(f"corr must be [M, {self.out_channels}, {self.h}, {self.w}]")
        if out is None:
            out = torch.empty(M, 128, self.h, self.w, dtype=torch.float16, device=self.device)
        self._cuda(out, torch.float16, "out")
        self._check(self.lib.dc_corr_encode(self._ctx, corr.data_ptr(), M, out.data_ptr(),
                                            _stream(stream)))
        return out

    def build_lookup_encode(self, ii, jj, coords: torch.Tensor,
                            corr: Optional[torch.Tensor] = None,
                            out: Optional[torch.Tensor] = None,
                            stream: Optional[torch.cuda.Stream] = None):
        """Fused correlation into `corr` [M, 196, h, w], then its encoding.
        Returns (out [M, 128, h, w] fp16, corr)."""
        ii, jj = self._edges(ii, jj)
        M = ii.numel()
        self._cuda(coords, torch.float32, "coords")
        if coords.shape != (M, 2, self.h, self.w):
            raise ValueError(f"coords must be [{M}, 2, {self.h}, {self.w}]")
        if corr is None:
            corr = torch.empty(M, self.out_channels, self.h, self.w, device=self.device)
        if out is None:
            out = torch.empty(M, 128, self.h, self.w, dtype=torch.float16, device=self.device)
        self._cuda(corr, torch.float32, "corr")
        self._cuda(out, torch.float16, "out")
        s = _stream(stream)
        for c0 in range(0, M, self.max_edges):
            m = min(self.max_edges, M - c0)
            self._check(self.lib.dc_build_lookup_encode(
                self._ctx, ii[c0].data_ptr(), jj[c0].data_ptr(), m, coords[c0].data_ptr(),
                corr[c0].data_ptr(), out[c0].data_ptr(), s))
        return out, corr

    def _project_args(self, poses, disps, intrinsics):
        self._cuda(poses, torch.float32, "poses")
        self._cuda(disps, torch.float32, "disps")
        self._cuda(intrinsics, torch.float32, "intrinsics")
        N = poses.shape[0]
        if poses.shape != (N, 7) or disps.shape != (N, self.h, self.w) or intrinsics.numel() != 4:
            raise ValueError(f"poses must be [N, 7], disps [N, {self.h}, {self.w}], intrinsics [4]")
        return N

    def project(self, poses: torch.Tensor, disps: torch.Tensor, intrinsics: torch.Tensor, ii, jj,
                coords: Optional[torch.Tensor] = None, valid: Optional[torch.Tensor] = None,
                stream: Optional[torch.cuda.Stream] = None):
        """Reproject every source pixel of each edge into frame jj (projmap_kernel,
        se3.cuh:118-177, plus the [M][hw][2] -> [M][2][hw] layout pass,
        main.cu:1135-1146).  Returns (coords [M, 2, h, w], valid [M, h, w])."""
        N = self._project_args(poses, disps, intrinsics)
        ii, jj = self._edges(ii, jj)
        M = ii.numel()
        if coords is None:
            coords = torch.empty(M, 2, self.h, self.w, device=self.device)
        if valid is None:
            valid = torch.empty(M, self.h, self.w, device=self.device)
        self._cuda(coords, torch.float32, "coords")
        self._cuda(valid, torch.float32, "valid")
        s = _stream(stream)
        for c0 in range(0, M, self.max_edges):
            m = min(self.max_edges, M - c0)
            self._check(self.lib.dc_project(self._ctx, poses.data_ptr(), disps.data_ptr(),
                                            intrinsics.data_ptr(), N, ii[c0].data_ptr(),
                                            jj[c0].data_ptr(), m, coords[c0].data_ptr(),
                                            valid[c0].data_ptr(), s))
        return coords, valid

    def project_build_and_lookup(self, poses: torch.Tensor, disps: torch.Tensor,
                                 intrinsics: torch.Tensor, ii, jj,
                                 out: Optional[torch.Tensor] = None,
                                 coords: Optional[torch.Tensor] = None,
                                 valid: Optional[torch.Tensor] = None,
                                 stream: Optional[torch.cuda.Stream] = None):
        """Reprojection, then the fused build + pyramid + lookup on those
        coordinates (the reference's per-batch steps 1-3, main.cu:2188-2201).
        Returns (out [M, 196, h, w], coords [M, 2, h, w], valid [M, h, w])."""
        N = self._project_args(poses, disps, intrinsics)
        ii, jj = self._edges(ii, jj)
        M = ii.numel()
        if coords is None:
            coords = torch.empty(M, 2, self.h, self.w, device=self.device)
        if valid is None:
            valid = torch.empty(M, self.h, self.w, device=self.device)
        if out is None:
            out = torch.empty(M, self.out_channels, self.h, self.w, device=self.device)
        for t, n in ((coords, "coords"), (valid, "valid"), (out, "out")):
            self._cuda(t, torch.float32, n)
        s = _stream(stream)
        for c0 in range(0, M, self.max_edges):
            m = min(self.max_edges, M - c0)
            self._check(self.lib.dc_project_build_and_lookup(
                self._ctx, poses.data_ptr(), disps.data_ptr(), intrinsics.data_ptr(), N,
                ii[c0].data_ptr(), jj[c0].data_ptr(), m, coords[c0].data_ptr(),
                valid[c0].data_ptr(), out[c0].data_ptr(), s))
        return out, coords, valid

    def scatter_mean(self, feats: torch.Tensor, ii, agg: Optional[torch.Tensor] = None,
                     stream: Optional[torch.cuda.Stream] = None):
        """GraphAgg scatter-mean (main.cu:2255-2294): the mean of feats[e] over the
        edges e of each distinct source keyframe ii[e], keyframes in ascending id
        order.  feats [E, ...] float32 on the device, ii a host sequence of E ids.
        Returns (agg [K, ...], kf_ids np.int32 [K])."""
        import numpy as np

        self._cuda(feats, torch.float32, "feats")
        ii_h = np.ascontiguousarray(np.asarray(ii, dtype=np.int32))
        E = feats.shape[0]
        if ii_h.shape != (E,):
            raise ValueError("ii must hold one keyframe id per row of feats")
        F = feats[0].numel() if E else 0
        if agg is None:
            agg = torch.empty((len(np.unique(ii_h)),) + tuple(feats.shape[1:]), device=self.device)
        self._cuda(agg, torch.float32, "agg")
        ids = np.empty(max(E, 1), np.int32)
        K = ctypes.c_int(0)
        self._check(self.lib.dc_scatter_mean(self._ctx, feats.data_ptr(), F,
                                             ii_h.ctypes.data, E, agg.data_ptr(),
                                             ids.ctypes.data, ctypes.byref(K), _stream(stream)))
        return agg[:K.value], ids[:K.value].copy()

    def gather_rows(self, src: torch.Tensor, idx, dst: Optional[torch.Tensor] = None,
                    stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        """dst[e] = src[idx[e]] (rows = src[0]'s elements) in one launch: the
        update step's per-edge `inps[ii[e]]` loads (main.cu:2215-2224).
        Out-of-range indices give zero rows."""
        self._cuda(src, torch.float32, "src")
        idx = torch.as_tensor(idx, dtype=torch.int32, device=self.device).contiguous()
        n = idx.numel()
        if dst is None:
            dst = torch.empty((n,) + tuple(src.shape[1:]), device=self.device)
        self._cuda(dst, torch.float32, "dst")
        F = src[0].numel()
        self._check(self.lib.dc_gather_rows(self._ctx, src.data_ptr(), F, src.shape[0],
                                            idx.data_ptr(), n, dst.data_ptr(), _stream(stream)))
        return dst

    def alt_lookup(self, ii, jj, coords: torch.Tensor, out: Optional[torch.Tensor] = None,
                   stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        """On-the-fly lookup from the pooled feature maps."""
        return self._edge_call(self.lib.dc_alt_lookup, ii, jj, coords, out, stream)

    # -- the reference's method names ------------------------------------------
    def build_correlation(self, i: int, j: int) -> None:
        """CudaDroid::build_correlation (main.cu:1500): fills corr_volume [hw, hw]
        and corr_pyramid[1..] [hw, h>>l, w>>l] for edge (i, j)."""
        vols = self.build_volume([i], [j])
        self.corr_volume = vols[0].view(self.hw, self.hw)
        self.corr_pyramid = [vols[0][0]] + [v[0] for v in vols[1:]]

    def sample_correlation(self, coords_2hw: torch.Tensor, corr_out: torch.Tensor) -> None:
        """CudaDroid::sample_correlation (main.cu:1529): coords [2,h,w] -> corr_out
        [196,h,w] from the volumes of the last build_correlation."""
        if self.corr_volume is None:
            raise L.DroidCorrError(L.DC_ERR_NOT_READY, "build_correlation was not called")
        vols = [self.corr_volume] + list(self.corr_pyramid[1:])
        self.lookup_single(vols, coords_2hw.view(2, self.h, self.w),
                           corr_out.view(self.out_channels, self.h, self.w))

    def batch_build_and_sample_correlation(self, batch_size: int, edge_start: int,
                                           coords_2hw: torch.Tensor,
                                           corr_out_196hw: torch.Tensor) -> None:
        """CudaDroid::batch_build_and_sample_correlation (main.cu:1555): edges
        ii_host/jj_host[edge_start : edge_start+batch_size], coords [M,2,h,w] ->
        corr_out [M,196,h,w]."""
        ii = self.ii_host[edge_start: edge_start + batch_size]
        jj = self.jj_host[edge_start: edge_start + batch_size]
        self.build_and_lookup(ii, jj, coords_2hw.view(batch_size, 2, self.h, self.w),
                              corr_out_196hw.view(batch_size, self.out_channels, self.h, self.w))
