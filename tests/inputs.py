"""Seeded synthetic inputs shared by the tests and the golden-fixture script.

numpy's PCG64 stream is the same on every machine, so a (shape, seed) pair
names one exact array here, on the GPU host and in the committed fixtures.
"""
import numpy as np


def normal(shape, sigma, seed):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal(shape, dtype=np.float32) * np.float32(sigma)).astype(np.float32)


def tensor_128x128_s8():
    """128x128 FP32 weights ~ N(0, 0.02^2) seed 0; 8 FP32 gradient samples ~ N(0, 1e-3^2) seed 1."""
    w = normal(16384, 0.02, 0)
    g = normal((8, 16384), 1e-3, 1)
    return w, g


def tie_heavy(N, S, seed):
    """Weights drawn from a handful of values (zeros, +-a, +-2a) and gradients of
    constant magnitude, so many groups tie at the N-th score."""
    rng = np.random.default_rng(seed)
    w = rng.choice(np.array([0.0, 0.01, -0.01, 0.02, -0.02, 0.0], np.float32), N).astype(np.float32)
    g = np.repeat(rng.choice(np.array([1e-3, -1e-3], np.float32), (1, N)), S, axis=0).astype(np.float32)
    return w, g


def outlier_columns(rows, cols, S, seed, frac=0.05, scale=10.0):
    """Weights N(0, 0.02^2), S gradients N(0, 1e-3^2) with `frac` of the input columns x`scale`."""
    w = normal(rows * cols, 0.02, seed)
    g = normal((S, rows, cols), 1e-3, seed + 1)
    rng = np.random.default_rng(seed + 2)
    hot = rng.choice(cols, max(1, int(cols * frac)), replace=False)
    g[:, :, hot] *= np.float32(scale)
    return w, g.reshape(S, rows * cols)


def to_bf16_bits(x):
    """Round-to-nearest-even FP32 -> BF16 bit patterns (uint16)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return r


def bf16_bits_to_f32(b):
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def write_safetensors(path, tensors):
    """Writes a .safetensors file: tensors is a list of (name, dtype, shape, raw bytes)."""
    import json
    import struct
    header, off, blobs = {}, 0, []
    for name, dtype, shape, raw in tensors:
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [off, off + len(raw)]}
        off += len(raw)
        blobs.append(raw)
    text = json.dumps(header, separators=(",", ":")).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(text)))
        f.write(text)
        for b in blobs:
            f.write(b)


def small_model(path):
    """Deterministic mixed-dtype checkpoint for the real-mode tb-prune runs."""
    q = normal(64 * 64, 0.02, 201)
    up = to_bf16_bits(normal(128 * 64, 0.02, 202))
    down = normal(64 * 128, 0.02, 203).astype(np.float16).view(np.uint16)
    norm = normal(62, 1.0, 204)
    head = normal(32 * 64, 0.02, 205)
    tokens = np.arange(10, dtype=np.int64)
    write_safetensors(path, [
        ("model.layers.0.self_attn.q_proj.weight", "F32", (64, 64), q.tobytes()),
        ("model.layers.0.mlp.up_proj.weight", "BF16", (128, 64), up.tobytes()),
        ("model.layers.0.mlp.down_proj.weight", "F16", (64, 128), down.tobytes()),
        ("model.norm.weight", "F32", (62,), norm.tobytes()),
        ("tokens", "I64", (10,), tokens.tobytes()),
        ("lm_head.weight", "F32", (32, 64), head.tobytes()),
    ])


MOCK_RUNS = {
    "oneshot_2of4": ["--mock-size", "16384", "--sparsity", "2:4"],
    "iterative_2of4": ["--mock-size", "16384", "--sparsity", "2:4", "--strategy", "Iterative"],
    "blockobs_2of4": ["--mock-size", "16384", "--sparsity", "2:4", "--strategy", "BlockOBS"],
    "magnitude_2of4": ["--mock-size", "16384", "--sparsity", "2:4", "--method", "Magnitude"],
    "oneshot_1of4": ["--mock-size", "8192", "--sparsity", "1:4"],
    "oneshot_2of8": ["--mock-size", "8192", "--sparsity", "2:8"],
    "oneshot_4of8": ["--mock-size", "8192", "--sparsity", "4:8"],
    "damping_10000": ["--mock-size", "10000", "--sparsity", "2:4", "--damping", "0.05"],
}


def activations(n, d, seed, frac=0.01, scale=20.0):
    """Calibration activations X [n][d] ~ N(0, 1) with a fraction of columns
    scaled (heavy-tail channels), rounded to BF16 and returned as FP32."""
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((n, d), dtype=np.float32)
    hot = rng.choice(d, max(1, int(d * frac)), replace=False)
    X[:, hot] *= np.float32(scale)
    return bf16_bits_to_f32(to_bf16_bits(X)).reshape(n, d)


def _tb_file(path, nm_n, nm_m, n_weights, mask_bytes, precision, seed, magic=0x31304254, payload=None):
    """A .tb file: the 4096-byte header, then `payload` bytes (default: FP32
    weights, or FP64 for precision 3, then the mask bytes)."""
    import struct
    rng = np.random.default_rng(seed)
    head = bytearray(4096)
    elem = 8 if precision == 3 else 4
    struct.pack_into("<IIIIQQQQB", head, 0, magic, 1, nm_n, nm_m, n_weights, mask_bytes,
                     4096, 4096 + elem * n_weights, precision)
    if payload is None:
        w = rng.standard_normal(n_weights).astype(np.float64 if elem == 8 else np.float32)
        payload = w.tobytes() + rng.integers(0, 256, mask_bytes, dtype=np.uint8).tobytes()
    with open(path, "wb") as f:
        f.write(bytes(head) + payload)


def merge_tree(root):
    """Two shard directories of .tb files for the .tbm merge, with the cases the
    merge has to get right: hidden names, suffixes inside names, duplicates
    (including a name reserved by a file whose header is bad), a truncated
    header, a wrong magic, an FP64 tensor and a short payload (offsets follow the
    headers, not the file sizes), quotes, backslashes and non-ASCII names, and
    files that are not .tb."""
    import os
    s1, s2 = os.path.join(root, "shard1"), os.path.join(root, "shard2")
    os.makedirs(s1)
    os.makedirs(s2)
    _tb_file(os.path.join(s1, "model.layers.0.self_attn.q_proj.weight.tb"), 2, 4, 96, 24, 0, 1)
    _tb_file(os.path.join(s1, "model.layers.0.mlp.down_proj.weight.tb"), 2, 8, 128, 16, 0, 2)
    _tb_file(os.path.join(s1, "lm_head.weight.tb"), 2, 4, 32, 8, 3, 3)
    _tb_file(os.path.join(s1, ".hidden.tb"), 1, 4, 16, 4, 1, 4)
    _tb_file(os.path.join(s1, "dup.tb"), 2, 4, 8, 2, 0, 5)
    _tb_file(os.path.join(s1, "bad_magic.tb"), 2, 4, 8, 2, 0, 6, magic=0x12345678)
    with open(os.path.join(s1, "zz_truncated.tb"), "wb") as f:
        f.write(bytes(range(100)))
    with open(os.path.join(s1, "model.tbm"), "wb") as f:
        f.write(b"not a container")
    with open(os.path.join(s1, "notes.txt"), "w") as f:
        f.write("ignored\n")
    _tb_file(os.path.join(s2, "model.layers.1.self_attn.q_proj.weight.tb"), 2, 4, 64, 16, 2, 7)
    _tb_file(os.path.join(s2, "dup.tb"), 2, 4, 8, 2, 0, 8)
    _tb_file(os.path.join(s2, "bad_magic.tb"), 2, 4, 8, 2, 0, 9)
    _tb_file(os.path.join(s2, 'we"ird\\name ü.tb'), 2, 4, 8, 2, 0, 10)
    _tb_file(os.path.join(s2, "emoji\U0001F600.tb"), 4, 8, 16, 2, 0, 11)
    _tb_file(os.path.join(s2, "x.tbm.tb"), 2, 4, 8, 2, 0, 12)
    _tb_file(os.path.join(s2, "a.tb.tb"), 2, 4, 8, 2, 0, 13)
    _tb_file(os.path.join(s2, "Upper.tb"), 2, 4, 8, 2, 0, 14)
    _tb_file(os.path.join(s2, "short_payload.tb"), 2, 4, 1000, 250, 0, 15, payload=bytes(40))
    os.makedirs(os.path.join(root, "empty"))
    return s1, s2


# tb-merge / merge_tbm.py runs over merge_tree(): (key, arguments, run from)
MERGE_RUNS = {
    "shards": (["--input", "./shard1/", "shard2", "missing_dir", "--output", "out/full/model.tbm"], "."),
    "reversed_arch": (["--input", "shard2", "shard1", "--output", "r.tbm",
                       "--architecture", 'mistral "7b" ü\\\U0001F600'], "."),
    "dot_input": (["--input", ".", "--output", "../dot/model.tbm"], "shard1"),
    "empty": (["--input", "empty", "--output", "e.tbm"], "."),
}


def layered_model(path, layers=3, seed=300):
    """A multi-tensor checkpoint for the pipelined real mode: per layer an F32
    q_proj (256 x 256), a BF16 up_proj (512 x 256), an F16 down_proj
    (256 x 512) and a norm vector (258 elements, not a multiple of M: tb-prune
    skips it at CORING), then an I64 tensor (skipped as non-float) and an F32
    lm_head - about 0.9 M weights per layer in the reference's dtypes."""
    tensors = []
    for k in range(layers):
        s = seed + 10 * k
        tensors.append((f"model.layers.{k}.self_attn.q_proj.weight", "F32", (256, 256),
                        normal(256 * 256, 0.02, s).tobytes()))
        tensors.append((f"model.layers.{k}.mlp.up_proj.weight", "BF16", (512, 256),
                        to_bf16_bits(normal(512 * 256, 0.02, s + 1)).tobytes()))
        tensors.append((f"model.layers.{k}.mlp.down_proj.weight", "F16", (256, 512),
                        normal(256 * 512, 0.02, s + 2).astype(np.float16).view(np.uint16).tobytes()))
        tensors.append((f"model.layers.{k}.input_layernorm.weight", "F32", (258,), normal(258, 1.0, s + 3).tobytes()))
    tensors.append(("position_ids", "I64", (16,), np.arange(16, dtype=np.int64).tobytes()))
    tensors.append(("lm_head.weight", "F32", (64, 256), normal(64 * 256, 0.02, seed + 99).tobytes()))
    write_safetensors(path, tensors)
