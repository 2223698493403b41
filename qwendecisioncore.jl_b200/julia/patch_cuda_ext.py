"""Route QwenDecisionCore.jl's CUDA extension through libqdc_b200.

The binding (QwenDecisionCoreB200Ext.jl) fills a hook table that the CUDA
extension reads; this file is the other half: the edits a maintainer makes
to the CUDA extension so that its row-kernel call sites go through that
table when it is set, and keep their own CUDA.jl kernels when it is not.

Each edit inserts lines of this project's own code next to an anchor line of
the reference file, checked by its SHA-256 (of the line without leading and
trailing white space), so no line of the reference is reproduced here and an
edit refuses a file whose anchor moved.  A site whose own kernel must stay
on the `else` side of the hook is bracketed by two insertions (`if ...
else` before, the hook call and `end` after).

    python patch_cuda_ext.py REFERENCE_DIR OUT_DIR   # patched copies of the ext/*.jl files
    python patch_cuda_ext.py REFERENCE_DIR --diff     # the same as a unified diff on stdout

Sites (reference ext/ files, lines of QwenDecisionCore.jl v0.1.0):
  cuda_workspace.jl:1    the hook table, B200Kernels = Ref{Any}(nothing)
  cuda_workspace.jl:65   native_forward_scope's finally: sync! reports device id errors
  cuda_workspace.jl:160  native_rms -> residual_rms!
  cuda_workspace.jl:199  native_residual_rms -> residual_rms!
  cuda_workspace.jl:333  native_gather -> gather!
  cuda_mlp.jl:67         native_mlp's SwiGLU -> swiglu!
  cuda_delta.jl:199-213  causal_depthwise + qk_normalize_kernel! -> delta_conv_norm_mixed!
  cuda_delta.jl:216-219  delta_gates_kernel! -> delta_gates!
  cuda_delta.jl:232-241  rms_gate_kernel! -> gated_rms!
  cuda_attention.jl:128-155  both prepare_head_kernel! launches -> qk_norm_rope_head_major!
  cuda_attention.jl:177-184  merge_gate_kernel! -> attn_gate!
  cuda_attention.jl:201-229  the last-token layer's prepare_head_kernel!s
  cuda_attention.jl:252-259  the last-token layer's merge_gate_kernel!
"""
import difflib
import hashlib
import os
import sys

class Edit:
    """Insert `text` before (where="before") or after (where="after") line
    `line` (1-based) of `file`, whose stripped content hashes to `sha256`."""

    def __init__(self, file, line, sha256, where, text):
        self.file, self.line, self.sha256, self.where, self.text = file, line, sha256, where, text


_END = "ba5ec51d07a4ac0e951608704431d59a02b21a4e951acc10505a8dc407c501ee"  # a call's closing parenthesis

EDITS = [
    # ---- cuda_workspace.jl
    Edit("ext/cuda_workspace.jl", 1, "cb54b29a7cf616bb746836766d1cddab012eaa7906294d94b55f571c718a5839",
         "before",
         "# libqdc_b200 hook table: QwenDecisionCoreB200Ext fills it on a compute capability 10.0\n"
         "# device; the row-kernel call sites below use it when it is set.\n"
         "const B200Kernels = Ref{Any}(nothing)\n"),
    Edit("ext/cuda_workspace.jl", 65, "cec5cf6354f133ab6e73826d5fbba572d6f66cbccfd8cf3476858bd41720a8c2",
         "after",
         "                B200Kernels[] === nothing || B200Kernels[].sync!()\n"),
    Edit("ext/cuda_workspace.jl", 160, "9ead8a1c415018c360a70844096f6bbbd816e27bcc88da289970cbbb53bf20c4",
         "before",
         "    B200Kernels[] === nothing ||\n"
         "        return B200Kernels[].residual_rms!(nothing, output, input, nothing, weight, eps; centered = centered)\n"),
    Edit("ext/cuda_workspace.jl", 199, "3cf5be18db976ea86b7ab7b2f61093f001f747d6639ffd98dd2928bd1c14162b",
         "before",
         "    if B200Kernels[] !== nothing\n"
         "        B200Kernels[].residual_rms!(residual, output, x, mixed, weight, eps)\n"
         "        return residual, output\n"
         "    end\n"),
    Edit("ext/cuda_workspace.jl", 333, "db6f4e8c26ce910a1cfd31f9b529050d71ba6819a277fcfc9e842c7a0552b99f",
         "before",
         "    B200Kernels[] === nothing ||\n"
         "        return B200Kernels[].gather!(scratch(Float32, (size(embedding, 1), length(ids))), embedding, ids)\n"),
    # ---- cuda_mlp.jl
    Edit("ext/cuda_mlp.jl", 67, "54aad7fcd1bbe4aeae63713a21e782072bf5fa620be2708ac7d97bf417e08a03", "before",
         "    B200Kernels[] === nothing ||\n"
         "        return QwenDecisionCore.native_linear(mlp.down, B200Kernels[].swiglu!(gated, projected))\n"),
    # ---- cuda_delta.jl: conv + q/k L2 norms, with v written into mixed's value rows
    Edit("ext/cuda_delta.jl", 199, "a87ce16218a111b6944326dd8273d7d6cf59ad45fdc1d65ce9d164c96cf35a51",
         "before", "    if B200Kernels[] === nothing\n"),
    Edit("ext/cuda_delta.jl", 213, _END, "after",
         "    else\n"
         "        mixed = scratch(Float32, (qkv_width, tokens))\n"
         "        query = scratch(Float32, (cfg.key_dim, cfg.key_heads, tokens))\n"
         "        key = scratch(Float32, size(query))\n"
         "        parts = Val(cld(cfg.key_dim, 32))\n"
         "        width = cfg.key_dim*cfg.key_heads\n"
         "        B200Kernels[].delta_conv_norm_mixed!(query, key, mixed, projected, attention.conv, cfg)\n"
         "    end\n"),
    Edit("ext/cuda_delta.jl", 216, "48f3cc1cf3401b3ac269abaa3cfdad94c15563b4dded84188259bf2eaea68afc",
         "before", "    if B200Kernels[] === nothing\n"),
    Edit("ext/cuda_delta.jl", 219, _END, "after",
         "    else\n"
         "        B200Kernels[].delta_gates!(beta, decay, projected, attention.a_decay, attention.dt_bias,\n"
         "                                   qkv_width + z_width)\n"
         "    end\n"),
    Edit("ext/cuda_delta.jl", 232, "9179b967c2013c30581ffcd33b7a588e52a6fd0a2db0306fc413d6c572b9c482",
         "before", "    if B200Kernels[] === nothing\n"),
    Edit("ext/cuda_delta.jl", 241, _END, "after",
         "    else\n"
         "        B200Kernels[].gated_rms!(gated, output, projected, attention.norm, cfg.eps; z_offset = qkv_width)\n"
         "    end\n"),
    # ---- cuda_attention.jl: q/k norm + RoPE (K expanded per query head) and the output gate
    Edit("ext/cuda_attention.jl", 128, "51f6a28bf50182ecde7f153c857c29bd4dc25acf397a93783fcdc421fad3716e",
         "before", "    if B200Kernels[] === nothing\n"),
    Edit("ext/cuda_attention.jl", 155, _END, "after",
         "    else\n"
         "        rope_cos, rope_sin = B200Kernels[].rope_device(cfg.rope_theta, cfg.rotary_dim, tokens)\n"
         "        B200Kernels[].qk_norm_rope_head_major!(q, qgate, attention.q_norm, cfg.eps, cfg.rotary_dim, rope_cos, rope_sin;\n"
         "                                               source_width = 2dim)\n"
         "        B200Kernels[].qk_norm_rope_head_major!(k, kp, attention.k_norm, cfg.eps, cfg.rotary_dim, rope_cos, rope_sin;\n"
         "                                               source_width = dim, row_offset = k_offset,\n"
         "                                               groups = heads ÷ kv_heads)\n"
         "    end\n"),
    Edit("ext/cuda_attention.jl", 177, "555da4b7a029eb53233544a96c24044fa7f2b16960c6146540c09ff385304a07",
         "before", "    if B200Kernels[] === nothing\n"),
    Edit("ext/cuda_attention.jl", 184, _END, "after",
         "    else\n"
         "        B200Kernels[].attn_gate!(merged, values, qgate)\n"
         "    end\n"),
    Edit("ext/cuda_attention.jl", 201, "fe39ef6ef2a316380a2154283307ad596d62cf41de802663a5363c6739181772",
         "before", "    if B200Kernels[] === nothing\n"),
    Edit("ext/cuda_attention.jl", 229, _END, "after",
         "    else\n"
         "        rope_cos, rope_sin = B200Kernels[].rope_device(cfg.rope_theta, cfg.rotary_dim, tokens)\n"
         "        B200Kernels[].qk_norm_rope_head_major!(q, qgate, attention.q_norm, cfg.eps, cfg.rotary_dim, rope_cos, rope_sin;\n"
         "                                               source_width = 2dim, offset = tokens - 1)\n"
         "        B200Kernels[].qk_norm_rope_head_major!(k, kvp, attention.k_norm, cfg.eps, cfg.rotary_dim, rope_cos, rope_sin;\n"
         "                                               source_width = dim, groups = heads ÷ kv_heads)\n"
         "    end\n"),
    Edit("ext/cuda_attention.jl", 252, "555da4b7a029eb53233544a96c24044fa7f2b16960c6146540c09ff385304a07",
         "before", "    if B200Kernels[] === nothing\n"),
    Edit("ext/cuda_attention.jl", 259, _END, "after",
         "    else\n"
         "        B200Kernels[].attn_gate!(merged, values, qgate)\n"
         "    end\n"),
]


def _digest(line):
    return hashlib.sha256(line.strip().encode()).hexdigest()


def patched(reference_dir):
    """{file: (original text, patched text)} for every file the edits touch.
    Raises ValueError when an anchor line does not hash as recorded."""
    out = {}
    for name in sorted({e.file for e in EDITS}):
        with open(os.path.join(reference_dir, name)) as f:
            original = f.read()
        lines = original.split("\n")
        # apply from the bottom so earlier line numbers stay valid
        for e in sorted((e for e in EDITS if e.file == name), key=lambda e: (e.line, e.where == "after"),
                        reverse=True):
            if not 1 <= e.line <= len(lines) or _digest(lines[e.line - 1]) != e.sha256:
                raise ValueError(f"{name}:{e.line}: anchor line differs from the one this edit was written for")
            at = e.line - 1 if e.where == "before" else e.line
            lines[at:at] = e.text.rstrip("\n").split("\n")
        out[name] = (original, "\n".join(lines))
    return out


def main(argv):
    if len(argv) != 3:
        raise SystemExit(__doc__)
    reference, target = argv[1], argv[2]
    files = patched(reference)
    if target == "--diff":
        for name, (old, new) in files.items():
            sys.stdout.writelines(difflib.unified_diff(old.splitlines(True), new.splitlines(True),
                                                       "a/" + name, "b/" + name))
        return
    for name, (_, new) in files.items():
        path = os.path.join(target, name)
        os.makedirs(os.path.dirname(path), exist_ok=True)
        with open(path, "w") as f:
            f.write(new)
        print(path)


if __name__ == "__main__":
    main(sys.argv)
