"""GGUF files and Gemma 3 loading straight to the device.

GgufFile follows the reference's reader (GgufFile::open / read_tensor_bytes /
find_tensor, src/gguf_loader.rs:142-252): magic "GGUF", version 2 or 3,
tensor and metadata counts, metadata key/value pairs (types 0-12, arrays
included), tensor infos (name, dims, type, offset), tensor data from the
header's end aligned to general.alignment (default 32).  The file is
memory-mapped and tensors are read as views of the map, with no copy on the
host.

load_gemma3 follows Gemma3Model::load_weights_from_gguf
(src/transformer4.rs:757-1010) for the tensors the CUDA engine keeps:
  token_embd.weight    BF16 as is; F16 / F32 -> BF16 (round to nearest even,
                       MatBf16::f32_to_bf16, src/autograd2.rs:709-719) on the
                       host; Q6_K -> BF16 on the GPU (rt_convert_q6k_to_bf16,
                       bit-exact with decode_q6k_to_f32 + f32s_to_bf16_and_drop)
  blk.N.attn_q/k/v, attn_output, ffn_gate/up/down
                       Q4_K as is (GGUF lists [in, out]: rows = dims[1]);
                       Q4_0 -> Q4_K on the GPU (rt_convert_q4_0_to_q4k,
                       bit-exact with decode_q4_0_to_q4mat + Q4KMat::from_q4mat)
  norms                F32 / F16, stored as 1 + gamma: gamma = value - 1
The engine streams Q4_K projections and ties the LM head to the embedding,
so a projection in another type, or an explicit output.weight, is refused
with GgufError (the reference keeps those as BF16 / a separate LM head).
Tensors outside the text model (vision tower, ...) are skipped, as there.
"""

import mmap
import re
import struct

import numpy as np

from ._lib import RT_FMT_BF16, RT_FMT_Q4K
from .model import Gemma3LayerWeights, Gemma3Weights

GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q8_0, GGML_Q4K, GGML_Q5K, GGML_Q6K, GGML_BF16 = 0, 1, 2, 8, 12, 13, 14, 30
# (bytes per block, elements per block): GgufType::block_info (src/gguf_loader.rs:112-124)
BLOCK_INFO = {GGML_F32: (4, 1), GGML_F16: (2, 1), GGML_BF16: (2, 1), GGML_Q4_0: (18, 32), GGML_Q8_0: (34, 32),
              GGML_Q4K: (144, 256), GGML_Q5K: (176, 256), GGML_Q6K: (210, 256)}
TYPE_NAMES = {GGML_F32: "F32", GGML_F16: "F16", GGML_Q4_0: "Q4_0", GGML_Q8_0: "Q8_0", GGML_Q4K: "Q4_K",
              GGML_Q5K: "Q5_K", GGML_Q6K: "Q6_K", GGML_BF16: "BF16"}

# metadata value types: 0 u8, 1 i8, 2 u16, 3 i16, 4 u32, 5 i32, 6 f32, 7 bool,
# 8 string, 9 array, 10 u64, 11 i64, 12 f64
_SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}


class GgufError(ValueError):
    pass


def byte_size(gtype, n_elements):
    """GgufType::byte_size (src/gguf_loader.rs:127-131), or None."""
    info = BLOCK_INFO.get(gtype)
    if info is None:
        return None
    bpb, epb = info
    return (n_elements + epb - 1) // epb * bpb


class GgufTensorInfo:
    def __init__(self, name, shape, gtype, offset):
        self.name, self.shape, self.gguf_type, self.data_offset = name, shape, gtype, offset

    def n_elements(self):
        n = 1
        for d in self.shape:
            n *= d
        return n


class GgufFile:
    """A parsed GGUF header over a memory map of the file."""

    def __init__(self, path):
        self.file_path = path
        self._f = open(path, "rb")
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        self.buf = np.frombuffer(self._mm, dtype=np.uint8)
        self._pos = 0
        if self._take(4) != b"GGUF":
            raise GgufError("not a GGUF file")
        self.version = self._scalar(4)
        if self.version < 2 or self.version > 3:
            raise GgufError(f"unsupported GGUF version {self.version}")
        n_tensors = self._scalar(10)
        n_kv = self._scalar(10)
        self.metadata = {}
        for _ in range(n_kv):
            key = self._string()
            self.metadata[key] = self._value(self._scalar(4))
        self.tensor_info = []
        for _ in range(n_tensors):
            name = self._string()
            n_dims = self._scalar(4)
            shape = [self._scalar(10) for _ in range(n_dims)]
            gtype = self._scalar(4)
            offset = self._scalar(10)
            self.tensor_info.append(GgufTensorInfo(name, shape, gtype, offset))
        align = int(self.metadata.get("general.alignment", 32))
        self.data_start = (self._pos + align - 1) // align * align

    def _take(self, n):
        if self._pos + n > len(self.buf):
            raise GgufError("truncated GGUF header")
        b = bytes(self.buf[self._pos:self._pos + n])
        self._pos += n
        return b

    def _scalar(self, vtype):
        fmt = _SCALAR[vtype]
        return struct.unpack(fmt, self._take(struct.calcsize(fmt)))[0]

    def _string(self):
        n = self._scalar(10)
        return self._take(n).decode("utf-8", errors="replace")

    def _value(self, vtype):
        if vtype in _SCALAR:
            return self._scalar(vtype)
        if vtype == 8:
            return self._string()
        if vtype == 9:
            etype = self._scalar(4)
            n = self._scalar(10)
            return [self._value(etype) for _ in range(n)]
        raise GgufError(f"unknown GGUF metadata type {vtype}")

    def find_tensor(self, name):
        for i, t in enumerate(self.tensor_info):
            if t.name == name:
                return i
        return None

    def tensor_bytes(self, idx):
        """The tensor's bytes, a view of the memory map (no copy)."""
        t = self.tensor_info[idx]
        n = byte_size(t.gguf_type, t.n_elements())
        if n is None:
            raise GgufError(f"unsupported gguf type {t.gguf_type} for tensor {t.name}")
        start = self.data_start + t.data_offset
        if start + n > len(self.buf):
            raise GgufError(f"tensor {t.name} runs past the end of the file")
        return self.buf[start:start + n]

    def close(self):
        self.buf = None
        if self._mm is not None:
            try:
                self._mm.close()
            except BufferError:  # a tensor view is still alive: the map goes with it
                pass
            self._mm = None
        if self._f is not None:
            self._f.close()
            self._f = None


def f32_to_bf16_bits(x):
    """MatBf16::f32_to_bf16 (src/autograd2.rs:709-719) over an array."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    out = ((b + np.uint32(0x7FFF) + ((b >> 16) & np.uint32(1))) >> 16).astype(np.uint16)
    nan = np.isnan(b.view(np.float32))
    out[nan] = ((b[nan] >> 16).astype(np.uint16) | np.uint16(0x0040))
    return out


def _norm(g, idx):
    t = g.tensor_info[idx]
    raw = g.tensor_bytes(idx)
    if t.gguf_type == GGML_F32:
        v = raw.view(np.float32).astype(np.float32)
    elif t.gguf_type == GGML_F16:
        v = raw.view(np.float16).astype(np.float32)
    else:
        raise GgufError(f"expected f32/f16 for norm tensor {t.name}")
    return (v - np.float32(1.0)).astype(np.float32)  # GGUF stores 1 + gamma


def _rows_cols(t):
    if len(t.shape) == 1:
        return 1, t.shape[0]
    if len(t.shape) == 2:
        return t.shape[1], t.shape[0]  # GGUF [cols, rows] -> [rows, cols]
    raise GgufError(f"unexpected shape rank {len(t.shape)} for {t.name}")


_PROJ = {"attn_q.weight": "q", "attn_k.weight": "k", "attn_v.weight": "v", "attn_output.weight": "o",
         "ffn_gate.weight": "gate", "ffn_up.weight": "up", "ffn_down.weight": "down"}
_NORMS = {"attn_norm.weight": "attn_norm", "post_attn_norm.weight": "post_attn_norm",
          "post_attention_norm.weight": "post_attn_norm", "ffn_pre_norm.weight": "pre_ffn_norm",
          "ffn_norm.weight": "pre_ffn_norm", "ffn_post_norm.weight": "post_ffn_norm",
          "post_ffw_norm.weight": "post_ffn_norm", "attn_q_norm.weight": "q_norm", "attn_k_norm.weight": "k_norm"}


def load_gemma3_weights(path, cfg, ctx):
    """Gemma3Weights whose projections and embedding are DeviceWeight handles
    on `ctx` (converted on the GPU where the file's type needs it) and whose
    norms are host arrays; CudaDecodeContext builds an engine from it."""
    from .ops import DeviceWeight, convert_q4_0_to_q4k, convert_q6k_to_bf16

    H, D, F = cfg.hidden_size, cfg.head_dim, cfg.intermediate_size
    q, kv = cfg.num_attention_heads * D, cfg.num_key_value_heads * D
    want = {"q": (q, H), "k": (kv, H), "v": (kv, H), "o": (H, q), "gate": (F, H), "up": (F, H), "down": (H, F)}
    g = GgufFile(path)
    made = []  # device weights, freed if loading fails
    try:
        layers = [dict() for _ in range(cfg.num_hidden_layers)]
        w = Gemma3Weights(cfg)
        for idx, t in enumerate(g.tensor_info):
            name = t.name
            if name == "token_embd.weight":
                rows, cols = _rows_cols(t)
                if (rows, cols) != (cfg.vocab_size, H):
                    raise GgufError(f"token_embd is [{rows}, {cols}], the config wants [{cfg.vocab_size}, {H}]")
                raw = g.tensor_bytes(idx)
                if t.gguf_type == GGML_BF16:
                    w.embed = DeviceWeight.upload(ctx, RT_FMT_BF16, raw.view(np.uint16), rows, cols)
                elif t.gguf_type == GGML_F16:
                    w.embed = DeviceWeight.upload(ctx, RT_FMT_BF16, f32_to_bf16_bits(raw.view(np.float16)), rows, cols)
                elif t.gguf_type == GGML_F32:
                    w.embed = DeviceWeight.upload(ctx, RT_FMT_BF16, f32_to_bf16_bits(raw.view(np.float32)), rows, cols)
                elif t.gguf_type == GGML_Q6K:
                    w.embed = convert_q6k_to_bf16(ctx, raw, rows, cols)
                else:
                    raise GgufError(f"token_embd type {TYPE_NAMES.get(t.gguf_type, t.gguf_type)} is not supported")
                made.append(w.embed)
            elif name == "output.weight":
                raise GgufError("an explicit output.weight (untied LM head) is not supported: "
                                "the engine's LM head is the embedding")
            elif name == "output_norm.weight":
                w.final_norm = _norm(g, idx)
            elif name.startswith("blk."):
                m = re.match(r"blk\.(\d+)\.(.+)$", name)
                if not m:
                    continue
                li, rest = int(m.group(1)), m.group(2)
                if li >= cfg.num_hidden_layers:
                    continue
                if rest in _NORMS:
                    layers[li][_NORMS[rest]] = _norm(g, idx)
                elif rest in _PROJ:
                    key = _PROJ[rest]
                    rows, cols = _rows_cols(t)
                    if (rows, cols) != want[key]:
                        raise GgufError(f"{name} is [{rows}, {cols}], the config wants {list(want[key])}")
                    raw = g.tensor_bytes(idx)
                    if t.gguf_type == GGML_Q4K:
                        dw = DeviceWeight.upload(ctx, RT_FMT_Q4K, raw, rows, cols)
                    elif t.gguf_type == GGML_Q4_0:
                        dw = convert_q4_0_to_q4k(ctx, raw, rows, cols)
                    else:
                        raise GgufError(f"{name}: projection type {TYPE_NAMES.get(t.gguf_type, t.gguf_type)} is "
                                        "not supported (the engine streams Q4_K; Q4_0 is converted)")
                    made.append(dw)
                    layers[li][key] = dw
        if w.embed is None or w.final_norm is None:
            raise GgufError("token_embd.weight and output_norm.weight are required")
        fields = ("q", "k", "v", "o", "gate", "up", "down", "attn_norm", "post_attn_norm", "pre_ffn_norm",
                  "post_ffn_norm", "q_norm", "k_norm")
        for i, L in enumerate(layers):
            missing = [f for f in fields if f not in L]
            if missing:
                raise GgufError(f"blk.{i}: missing {', '.join(missing)}")
            w.layers.append(Gemma3LayerWeights(**{f: L[f] for f in fields}))
        return w
    except Exception:
        for dw in made:
            dw.free()
        raise
    finally:
        g.close()


def load_gemma3(path, cfg, max_ctx, ctx=None):
    """A CudaDecodeContext for the Gemma 3 model in GGUF file `path` (`cfg`
    gives the hyperparameters, as the reference's caller does)."""
    from .decode import CudaDecodeContext
    from .ops import Context

    ctx = ctx or Context(0)
    w = load_gemma3_weights(path, cfg, ctx)
    return CudaDecodeContext(w, max_ctx, ctx)


def _pack_value(vtype, value):
    if vtype in _SCALAR:
        return struct.pack(_SCALAR[vtype], value)
    if vtype == 8:
        b = value.encode("utf-8")
        return struct.pack("<Q", len(b)) + b
    if vtype == 9:
        etype, items = value
        return struct.pack("<IQ", etype, len(items)) + b"".join(_pack_value(etype, v) for v in items)
    raise GgufError(f"unknown GGUF metadata type {vtype}")


def write_gguf(path, tensors, metadata=(), alignment=32, version=3):
    """Write a GGUF file (the layout GgufFile reads).  tensors: (name, dims in
    GGUF order, type, bytes); metadata: (key, type, value), an array's value
    being (element type, items).  A general.alignment entry, if any, must
    match `alignment`."""
    meta = list(metadata)
    head = [b"GGUF", struct.pack("<IQQ", version, len(tensors), len(meta))]
    for key, vtype, value in meta:
        kb = key.encode("utf-8")
        head.append(struct.pack("<Q", len(kb)) + kb + struct.pack("<I", vtype) + _pack_value(vtype, value))
    offset = 0
    blobs = []
    for name, dims, gtype, data in tensors:
        data = np.ascontiguousarray(data).view(np.uint8).reshape(-1).tobytes()
        n = 1
        for d in dims:
            n *= d
        if byte_size(gtype, n) != len(data):
            raise GgufError(f"{name}: {len(data)} bytes for {dims} of type {gtype}")
        nb = name.encode("utf-8")
        head.append(struct.pack("<Q", len(nb)) + nb + struct.pack("<I", len(dims)) +
                    b"".join(struct.pack("<Q", d) for d in dims) + struct.pack("<IQ", gtype, offset))
        pad = (-len(data)) % alignment
        blobs.append(data + b"\0" * pad)
        offset += len(data) + pad
    header = b"".join(head)
    header += b"\0" * ((-len(header)) % alignment)
    with open(path, "wb") as f:
        f.write(header)
        for b in blobs:
            f.write(b)
