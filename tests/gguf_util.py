"""Write synthetic SigLIP2 checkpoints (b2q.synth) as GGUF files with gguf-py,
the package the reference's converter uses (scripts/convert_siglip2_to_gguf.py)."""
import numpy as np


def write_checkpoint(path, ck, f16_weights=None, f32_weights=None, extra=None):
    """Q8_0 tensors as Q8_0 blocks, F32 tensors as F32.  f16_weights /
    f32_weights map projection names to weights to store unquantized as F16 /
    F32 instead (F16 is the converter's fallback for ffn_down, whose K = 4304
    is not a multiple of 32).  extra: more name -> array entries (e.g. the
    [1]-shaped logit scalars)."""
    import gguf
    w = gguf.GGUFWriter(str(path), "siglip2")
    w.add_string("general.name", "synthetic siglip2")
    w.add_uint32("siglip2.vision.block_count", ck.cfg.n_layer)
    w.add_array("siglip2.test.tags", ["a", "bc"])
    f16_weights = f16_weights or {}
    f32_weights = f32_weights or {}
    for name, arr in ck.tensors.items():
        if name in f16_weights:
            w.add_tensor(name, np.ascontiguousarray(f16_weights[name].astype(np.float16)))
        elif name in f32_weights:
            w.add_tensor(name, np.ascontiguousarray(f32_weights[name].astype(np.float32)))
        elif name in ck.q8_shapes:
            n, _, kp = ck.q8_shapes[name]
            w.add_tensor(name, np.ascontiguousarray(arr).reshape(n, kp // 32 * 34),
                         raw_dtype=gguf.GGMLQuantizationType.Q8_0)
        else:
            w.add_tensor(name, np.ascontiguousarray(arr, np.float32))
    for name, arr in (extra or {}).items():
        w.add_tensor(name, np.ascontiguousarray(arr))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
