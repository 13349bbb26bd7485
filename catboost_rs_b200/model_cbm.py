"""The CatBoost binary model format (.cbm) for the oblivious models this package trains.

The reference reads and writes this format in crates/cb-model/src/cbm.rs
(save_cbm :635, decode_cbm :1062); it is upstream CatBoost's model file:

- framing: the 4 bytes ``CBM1``, a little-endian u32 with the byte length of
  the core, then the core, a FlatBuffers buffer whose root is ``TModelCore``
  (cbm.rs:1-20).  Model parts after the core (CTR tables, text and embedding
  models) are not produced by this package; a file carrying them is rejected.
- ``TModelCore``: ``FormatVersion`` (the string ``FlabuffersModel_v1``,
  spelled as upstream spells it), ``ModelTrees``, ``InfoMap`` (string key /
  value pairs) and ``ModelPartIds``.
- ``TModelTrees``: ``ApproxDimension``; ``TreeSplits`` (per level of every
  tree, the split's index in the model's binary-feature list: every float
  feature's borders in feature order, then every one-hot feature's values);
  ``TreeSizes`` (depth per tree); ``TreeStartOffsets`` (each tree's first
  entry in TreeSplits); ``FloatFeatures`` (borders as f32 with the NaN
  treatment); ``CatFeatures`` and ``OneHotFeatures`` (per one-hot feature its
  category hash values); ``LeafValues`` (all trees, leaf-major,
  ``leaf * dim + d``) and ``LeafWeights``; ``Scale`` / ``Bias`` /
  ``MultiBias``.

The FlatBuffers wire format is restated here from its published description
(little-endian; a table starts with a signed 32-bit offset back to its
vtable; a vtable is u16 vtable size, u16 table size, then one u16 per field
with the field's offset in the table, 0 when absent; references to tables,
vectors and strings are unsigned 32-bit offsets forward from the referring
position; a vector or string is a u32 count followed by its elements, a
string also by a NUL).  The reader checks every offset, count and alignment
against the buffer, like the reference's verifying decoder, and raises
ValueError on anything malformed.  Field slots come from upstream's
model.fbs schema, which the reference uses through generated code.

Scope: oblivious (symmetric) trees over float features and one-hot
categorical features -- what ObliviousModel and MultiClassModel hold.
Non-symmetric trees, CTR features, text and embedding features are rejected
with ValueError, as model.json rejects what it cannot represent.
"""
from __future__ import annotations

import struct
from typing import List, Optional, Tuple, Union

import numpy as np

from .boosting import MultiClassModel, ObliviousModel
from .cat_hash import cat_feature_hash

MAGIC = b"CBM1"
FORMAT_VERSION = "FlabuffersModel_v1"
_FLT_MAX = float(np.finfo(np.float32).max)

# vtable slots (byte offsets inside the vtable) of the tables used here
_CORE = {"FormatVersion": 4, "ModelTrees": 6, "InfoMap": 8, "ModelPartIds": 10}
_TREES = {"ApproxDimension": 4, "TreeSplits": 6, "TreeSizes": 8, "TreeStartOffsets": 10, "CatFeatures": 12,
          "FloatFeatures": 14, "OneHotFeatures": 16, "CtrFeatures": 18, "LeafValues": 20, "LeafWeights": 22,
          "NonSymmetricStepNodes": 24, "NonSymmetricNodeIdToLeafId": 26, "TextFeatures": 28,
          "EstimatedFeatures": 30, "Scale": 32, "Bias": 34, "MultiBias": 36, "RepackedBins": 38,
          "EmbeddingFeatures": 40}
_FLOAT = {"HasNans": 4, "Index": 6, "FlatIndex": 8, "Borders": 10, "FeatureId": 12, "NanValueTreatment": 14}
_CAT = {"Index": 4, "FlatIndex": 6, "FeatureId": 8, "UsedInModel": 10}
_ONEHOT = {"Index": 4, "Values": 6, "StringValues": 8}
_KV = {"Key": 4, "Value": 6}
_NAN_TREATMENT = {0: "AsIs", 1: "AsFalse", 2: "AsTrue"}


# ---------------------------------------------------------------------------
# reading
# ---------------------------------------------------------------------------

class _Table:
    """One FlatBuffers table of a verified buffer."""

    def __init__(self, buf: bytes, pos: int):
        self.buf = buf
        self.pos = pos
        _need(buf, pos, 4, 4, "table")
        vt = pos - struct.unpack_from("<i", buf, pos)[0]
        _need(buf, vt, 4, 2, "vtable")
        self.vt_size, self.size = struct.unpack_from("<HH", buf, vt)
        if self.vt_size < 4 or self.vt_size % 2:
            raise ValueError(f"malformed vtable size {self.vt_size} at {vt}")
        _need(buf, vt, self.vt_size, 2, "vtable")
        _need(buf, pos, max(self.size, 4), 1, "table body")
        self.vt = vt

    def _field(self, slot: int) -> int:
        """Absolute position of the field in slot, or 0 when absent."""
        if slot >= self.vt_size:
            return 0
        off = struct.unpack_from("<H", self.buf, self.vt + slot)[0]
        if off and off >= max(self.size, 4):
            raise ValueError(f"field offset {off} outside its table of {self.size} bytes")
        return self.pos + off if off else 0

    def has(self, slot: int) -> bool:
        return self._field(slot) != 0

    def scalar(self, slot: int, fmt: str, default):
        p = self._field(slot)
        if not p:
            return default
        size = struct.calcsize("<" + fmt)
        _need(self.buf, p, size, size, "scalar field")
        return struct.unpack_from("<" + fmt, self.buf, p)[0]

    def _target(self, slot: int) -> int:
        p = self._field(slot)
        if not p:
            return 0
        _need(self.buf, p, 4, 4, "offset field")
        return p + struct.unpack_from("<I", self.buf, p)[0]

    def vector(self, slot: int, fmt: str) -> Optional[np.ndarray]:
        t = self._target(slot)
        if not t:
            return None
        size = struct.calcsize("<" + fmt)
        _need(self.buf, t, 4, 4, "vector")
        n = struct.unpack_from("<I", self.buf, t)[0]
        _need(self.buf, t + 4, n * size, size, "vector body")
        return np.frombuffer(self.buf, dtype=np.dtype("<" + fmt), count=n, offset=t + 4).copy()

    def vector_len(self, slot: int) -> int:
        t = self._target(slot)
        if not t:
            return 0
        _need(self.buf, t, 4, 4, "vector")
        return struct.unpack_from("<I", self.buf, t)[0]

    def string(self, slot: int) -> Optional[str]:
        t = self._target(slot)
        if not t:
            return None
        _need(self.buf, t, 4, 4, "string")
        n = struct.unpack_from("<I", self.buf, t)[0]
        _need(self.buf, t + 4, n + 1, 1, "string body")
        if self.buf[t + 4 + n] != 0:
            raise ValueError("string without its terminating NUL")
        return self.buf[t + 4:t + 4 + n].decode("utf-8")

    def table(self, slot: int) -> Optional["_Table"]:
        t = self._target(slot)
        return _Table(self.buf, t) if t else None

    def tables(self, slot: int) -> Optional[List["_Table"]]:
        t = self._target(slot)
        if not t:
            return None
        _need(self.buf, t, 4, 4, "vector")
        n = struct.unpack_from("<I", self.buf, t)[0]
        _need(self.buf, t + 4, 4 * n, 4, "vector body")
        out = []
        for k in range(n):
            p = t + 4 + 4 * k
            out.append(_Table(self.buf, p + struct.unpack_from("<I", self.buf, p)[0]))
        return out


def _need(buf: bytes, pos: int, size: int, align: int, what: str) -> None:
    if pos < 0 or size < 0 or pos + size > len(buf):
        raise ValueError(f"{what} at {pos} (+{size}) runs past the {len(buf)}-byte buffer")
    if align > 1 and pos % align:
        raise ValueError(f"{what} at {pos} is not {align}-byte aligned")


def _core_of(data: bytes) -> bytes:
    if data[0:4] != MAGIC:
        raise ValueError("bad .cbm magic (expected CBM1)")
    if len(data) < 8:
        raise ValueError("truncated .cbm header")
    n = struct.unpack_from("<I", data, 4)[0]
    if 8 + n > len(data):
        raise ValueError(f"declared core size {n} exceeds the {len(data) - 8} bytes after the header")
    if 8 + n < len(data):
        raise ValueError("model parts after the core (CTR / text / embedding data) are not supported")
    return bytes(data[8:8 + n])


def read_core(data: bytes) -> dict:
    """The fields of a .cbm file's TModelCore as plain Python / numpy values
    (absent fields omitted); raises ValueError on a malformed buffer."""
    core = _core_of(data)
    _need(core, 0, 4, 4, "root offset")
    root = _Table(core, struct.unpack_from("<I", core, 0)[0])
    out = {"FormatVersion": root.string(_CORE["FormatVersion"])}
    info = root.tables(_CORE["InfoMap"])
    if info is not None:
        out["InfoMap"] = {kv.string(_KV["Key"]): kv.string(_KV["Value"]) for kv in info}
    trees = root.table(_CORE["ModelTrees"])
    if trees is None:
        raise ValueError("the core has no ModelTrees")
    t = {"ApproxDimension": trees.scalar(_TREES["ApproxDimension"], "i", 0),
         "Scale": trees.scalar(_TREES["Scale"], "d", 1.0),
         "Bias": trees.scalar(_TREES["Bias"], "d", 0.0)}
    for name, fmt in (("TreeSplits", "i"), ("TreeSizes", "i"), ("TreeStartOffsets", "i"),
                      ("LeafValues", "d"), ("LeafWeights", "d"), ("MultiBias", "d")):
        v = trees.vector(_TREES[name], fmt)
        if v is not None:
            t[name] = v
    floats = []
    for f in trees.tables(_TREES["FloatFeatures"]) or []:
        floats.append({"HasNans": bool(f.scalar(_FLOAT["HasNans"], "B", 0)),
                       "Index": f.scalar(_FLOAT["Index"], "i", -1),
                       "FlatIndex": f.scalar(_FLOAT["FlatIndex"], "i", -1),
                       "Borders": f.vector(_FLOAT["Borders"], "f"),
                       "FeatureId": f.string(_FLOAT["FeatureId"]),
                       "NanValueTreatment": _NAN_TREATMENT.get(f.scalar(_FLOAT["NanValueTreatment"], "b", 0),
                                                               "AsIs")})
    t["FloatFeatures"] = floats
    t["CatFeatures"] = [{"Index": c.scalar(_CAT["Index"], "i", -1), "FlatIndex": c.scalar(_CAT["FlatIndex"], "i", -1),
                         "FeatureId": c.string(_CAT["FeatureId"]),
                         "UsedInModel": bool(c.scalar(_CAT["UsedInModel"], "B", 1))}
                        for c in trees.tables(_TREES["CatFeatures"]) or []]
    t["OneHotFeatures"] = [{"Index": o.scalar(_ONEHOT["Index"], "i", -1), "Values": o.vector(_ONEHOT["Values"], "i")}
                           for o in trees.tables(_TREES["OneHotFeatures"]) or []]
    # sections this package does not model count only when non-empty
    # (upstream writes empty vectors for them)
    for name in ("CtrFeatures", "NonSymmetricStepNodes", "NonSymmetricNodeIdToLeafId", "TextFeatures",
                 "EstimatedFeatures", "EmbeddingFeatures"):
        if trees.vector_len(_TREES[name]):
            t["Has" + name] = True
    out["ModelTrees"] = t
    return out


def from_core(core: dict) -> Union[ObliviousModel, MultiClassModel]:
    """A model from read_core's fields.  One-hot features become trailing
    "features" F, F+1, ... whose bins are the listed category hashes, as
    MultiClassModel stores them (cat_values = each feature's hashes)."""
    if core.get("FormatVersion") != FORMAT_VERSION:
        raise ValueError(f"unsupported FormatVersion {core.get('FormatVersion')!r}")
    t = core["ModelTrees"]
    for name in ("CtrFeatures", "NonSymmetricStepNodes", "NonSymmetricNodeIdToLeafId", "TextFeatures",
                 "EstimatedFeatures", "EmbeddingFeatures"):
        if t.get("Has" + name):
            raise ValueError(f"{name} are not supported (oblivious float / one-hot models only)")
    if t["Scale"] != 1.0:
        raise ValueError(f"scale {t['Scale']} is not supported")
    dim = max(1, int(t["ApproxDimension"]))
    floats = sorted(t["FloatFeatures"], key=lambda f: f["Index"])
    if [f["Index"] for f in floats] != list(range(len(floats))):
        raise ValueError("float feature indices are not 0..F-1")
    borders = [np.asarray(f["Borders"] if f["Borders"] is not None else [], dtype=np.float32).astype(np.float64)
               for f in floats]
    onehots = sorted(t["OneHotFeatures"], key=lambda o: o["Index"])
    cat_values = [np.asarray(o["Values"] if o["Values"] is not None else [], dtype=np.int64) for o in onehots]
    # binary-feature list: float borders, then one-hot values
    bins: List[Tuple[int, int]] = [(f, b) for f in range(len(borders)) for b in range(len(borders[f]))]
    bins += [(len(borders) + k, v) for k in range(len(onehots)) for v in range(len(cat_values[k]))]
    splits = t.get("TreeSplits", np.zeros(0, np.int32))
    sizes = t.get("TreeSizes", np.zeros(0, np.int32))
    starts = t.get("TreeStartOffsets", np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(np.int32))
    if len(sizes) == 0:
        raise ValueError("no trees")
    if len(set(int(s) for s in sizes)) != 1:
        raise ValueError("trees of different depths are not supported")
    T, D = len(sizes), int(sizes[0])
    L = 1 << D
    sf = np.zeros((T, D), dtype=np.int32)
    sb = np.zeros((T, D), dtype=np.int32)
    for k in range(T):
        s0 = int(starts[k])
        if s0 < 0 or s0 + D > len(splits):
            raise ValueError(f"tree {k}'s splits run past TreeSplits")
        for l in range(D):
            g = int(splits[s0 + l])
            if g < 0 or g >= len(bins):
                raise ValueError(f"split index {g} outside the {len(bins)} binary features")
            sf[k, l], sb[k, l] = bins[g]
    lv = np.asarray(t.get("LeafValues", np.zeros(0)), dtype=np.float64)
    if lv.size != T * L * dim:
        raise ValueError(f"{lv.size} leaf values, expected {T * L * dim}")
    lw = np.asarray(t.get("LeafWeights", np.zeros(T * L)), dtype=np.float64)
    if lw.size != T * L:
        lw = np.zeros(T * L)
    lv = lv.reshape(T, L, dim)
    multi_bias = t.get("MultiBias")
    # the bias lives in MultiBias (one per dimension); Bias is the older scalar slot
    bias = np.asarray(multi_bias if multi_bias is not None and len(multi_bias) else [t["Bias"]] * dim,
                      dtype=np.float64)
    if bias.size != dim:
        raise ValueError(f"{bias.size} bias values for {dim} dimensions")
    if dim == 1 and not onehots:
        m = ObliviousModel(borders, sf, sb, lv[:, :, 0], float(bias[0]))
    else:
        if np.any(bias != 0.0):
            raise ValueError("a bias on a multi-dimensional or one-hot model is not supported")
        m = MultiClassModel(borders, sf, sb, lv, cat_values=cat_values or None)
        m.cat_values_are_hashes = bool(onehots)
    m.leaf_weights = lw.reshape(T, L)
    m.info = dict(core.get("InfoMap") or {})
    return m


def load_cbm(path: str) -> Union[ObliviousModel, MultiClassModel]:
    with open(path, "rb") as fh:
        return from_cbm_bytes(fh.read())


def from_cbm_bytes(data: bytes) -> Union[ObliviousModel, MultiClassModel]:
    return from_core(read_core(data))


# ---------------------------------------------------------------------------
# writing
# ---------------------------------------------------------------------------
# Objects are laid out front to back: a table's vtable, then the table, then
# the objects it refers to, so every reference is a forward (unsigned)
# offset.  Every scalar sits at a multiple of its size from the start of the
# core (which the 8-byte header keeps 8-aligned in the file).

class _Vec:
    def __init__(self, fmt: str, values):
        self.fmt, self.values = fmt, list(values)


class _Str:
    def __init__(self, text: str):
        self.text = text


class _Tab:
    """fields: (slot, kind, value); kind is a struct format for inline
    scalars or "ref" for a _Vec / _Str / _Tab / list of _Tab."""

    def __init__(self, fields):
        self.fields = [f for f in fields if f[2] is not None]


class _Writer:
    def __init__(self):
        self.b = bytearray()

    def _pad_to(self, align: int, extra: int = 0) -> None:
        while (len(self.b) + extra) % align:
            self.b.append(0)

    def _patch_ref(self, at: int, target: int) -> None:
        struct.pack_into("<I", self.b, at, target - at)

    def emit(self, obj) -> int:
        if isinstance(obj, _Str):
            data = obj.text.encode("utf-8")
            self._pad_to(4)
            pos = len(self.b)
            self.b += struct.pack("<I", len(data)) + data + b"\0"
            return pos
        if isinstance(obj, _Vec):
            size = struct.calcsize("<" + obj.fmt)
            self._pad_to(max(size, 4), 4 if size == 8 else 0)  # elements aligned to their size
            pos = len(self.b)
            self.b += struct.pack("<I", len(obj.values))
            self.b += struct.pack("<%d%s" % (len(obj.values), obj.fmt), *obj.values)
            return pos
        if isinstance(obj, list):  # vector of tables
            self._pad_to(4)
            pos = len(self.b)
            self.b += struct.pack("<I", len(obj)) + bytes(4 * len(obj))
            for k, t in enumerate(obj):
                self._patch_ref(pos + 4 + 4 * k, self.emit(t))
            return pos
        return self._emit_table(obj)

    def _emit_table(self, tab: _Tab) -> int:
        # inline layout: the soffset, then 8-, 4- and 1-byte fields, each at a
        # multiple of its size (the table starts 8-aligned)
        sized = []
        for slot, kind, value in tab.fields:
            size = 4 if kind == "ref" else struct.calcsize("<" + kind)
            sized.append((size, slot, kind, value))
        place, off = {}, 4
        for want in (8, 4, 2, 1):
            for size, slot, kind, value in sized:
                if size != want:
                    continue
                off = (off + size - 1) // size * size
                place[slot] = off
                off += size
        tbl_size = (off + 3) // 4 * 4
        n_slots = max([(slot - 4) // 2 + 1 for slot, _, _ in tab.fields] or [0])
        vt = struct.pack("<HH", 4 + 2 * n_slots, tbl_size)
        vt += b"".join(struct.pack("<H", place.get(4 + 2 * k, 0)) for k in range(n_slots))
        self._pad_to(2)
        vt_pos = len(self.b)
        self.b += vt
        self._pad_to(8)
        pos = len(self.b)
        self.b += bytes(tbl_size)
        struct.pack_into("<i", self.b, pos, pos - vt_pos)
        refs = []
        for size, slot, kind, value in sized:
            if kind == "ref":
                refs.append((pos + place[slot], value))
            else:
                struct.pack_into("<" + kind, self.b, pos + place[slot], value)
        for at, child in refs:
            self._patch_ref(at, self.emit(child))
        return pos


def _nan_treatment(borders) -> Tuple[bool, int]:
    b = list(borders)
    if b and b[0] == -_FLT_MAX:
        return True, 1  # AsFalse: NaN compares below every border (nan_mode Min)
    if b and b[-1] == _FLT_MAX:
        return True, 2  # AsTrue (nan_mode Max)
    return False, 0


def to_cbm_bytes(model: Union[ObliviousModel, MultiClassModel], info: Optional[dict] = None) -> bytes:
    """The model as a .cbm file (header + TModelCore).  info: extra string
    InfoMap entries.  One-hot categories are written as their CatFeatureHash
    (models loaded from a .cbm already hold hashes and keep them)."""
    borders = [np.asarray(b, dtype=np.float64) for b in model.borders]
    F = len(borders)
    for f, b in enumerate(borders):
        if np.any(b.astype(np.float32).astype(np.float64) != b):
            raise ValueError(f"feature {f} has borders that are not f32 values (the format stores f32)")
    sf = np.asarray(model.split_feature, dtype=np.int64)
    sb = np.asarray(model.split_bin, dtype=np.int64)
    T, D = sf.shape
    L = 1 << D
    lv = np.asarray(model.leaf_values, dtype=np.float64)
    dim = 1 if lv.ndim == 2 else lv.shape[2]
    lv = lv.reshape(T, L, dim)
    cats = list(getattr(model, "cat_values", None) or [])
    if (sf >= F + len(cats)).any():
        raise ValueError("a split refers to a feature the model does not list")
    if getattr(model, "cat_values_are_hashes", False):
        hashes = [[int(v) & 0xFFFFFFFF for v in c] for c in cats]
    else:
        hashes = [[cat_feature_hash(v) for v in c] for c in cats]
    # binary-feature index of every (feature, bin)
    first = np.concatenate([[0], np.cumsum([len(b) for b in borders] + [len(h) for h in hashes])]).astype(np.int64)
    splits = []
    for t in range(T):
        for l in range(D):
            f, b = int(sf[t, l]), int(sb[t, l])
            width = len(borders[f]) if f < F else len(hashes[f - F])
            if not 0 <= b < width:
                raise ValueError(f"tree {t} level {l}: bin {b} outside feature {f}'s {width} bins")
            splits.append(int(first[f] + b))
    floats = []
    for f, b in enumerate(borders):
        has_nans, treat = _nan_treatment(b)
        floats.append(_Tab([(_FLOAT["HasNans"], "B", int(has_nans)), (_FLOAT["Index"], "i", f),
                            (_FLOAT["FlatIndex"], "i", f), (_FLOAT["Borders"], "ref", _Vec("f", b)),
                            (_FLOAT["NanValueTreatment"], "b", treat)]))
    cat_tabs = [_Tab([(_CAT["Index"], "i", k), (_CAT["FlatIndex"], "i", F + k), (_CAT["UsedInModel"], "B", 1)])
                for k in range(len(hashes))]
    onehot_tabs = [_Tab([(_ONEHOT["Index"], "i", k),
                         (_ONEHOT["Values"], "ref", _Vec("i", [h - (1 << 32) if h >= 1 << 31 else h for h in hv]))])
                   for k, hv in enumerate(hashes)]
    bias = float(getattr(model, "bias", 0.0) or 0.0)
    weights = getattr(model, "leaf_weights", None)
    lw = np.zeros(T * L) if weights is None else np.asarray(weights, dtype=np.float64).reshape(-1)
    trees = _Tab([
        (_TREES["ApproxDimension"], "i", dim),
        (_TREES["TreeSplits"], "ref", _Vec("i", splits)),
        (_TREES["TreeSizes"], "ref", _Vec("i", [D] * T)),
        (_TREES["TreeStartOffsets"], "ref", _Vec("i", [D * t for t in range(T)])),
        (_TREES["CatFeatures"], "ref", cat_tabs or None),
        (_TREES["FloatFeatures"], "ref", floats),
        (_TREES["OneHotFeatures"], "ref", onehot_tabs or None),
        (_TREES["LeafValues"], "ref", _Vec("d", lv.reshape(-1))),
        (_TREES["LeafWeights"], "ref", _Vec("d", lw)),
        (_TREES["MultiBias"], "ref", _Vec("d", [bias] * dim)),
    ])
    entries = dict(info or {})
    if dim > 1 and "class_params" not in entries:
        entries["class_params"] = '{"class_to_label":[%s]}' % ",".join("%d" % k for k in range(dim))
    kv = [_Tab([(_KV["Key"], "ref", _Str(k)), (_KV["Value"], "ref", _Str(str(entries[k])))])
          for k in sorted(entries)]  # a sorted map: readers may binary-search it
    core = _Tab([(_CORE["FormatVersion"], "ref", _Str(FORMAT_VERSION)),
                 (_CORE["ModelTrees"], "ref", trees),
                 (_CORE["InfoMap"], "ref", kv)])
    w = _Writer()
    w.b += bytes(4)  # root offset
    w._patch_ref(0, w.emit(core))
    w._pad_to(8)
    body = bytes(w.b)
    return MAGIC + struct.pack("<I", len(body)) + body


def save_cbm(model: Union[ObliviousModel, MultiClassModel], path: str, info: Optional[dict] = None) -> None:
    with open(path, "wb") as fh:
        fh.write(to_cbm_bytes(model, info))
