# QwenDecisionCoreB200Ext -- binds libqdc_b200.so into QwenDecisionCore.jl.
#
# A package extension of QwenDecisionCore.jl (declare it in Project.toml
# [extensions] next to QwenDecisionCoreCUDAExt, triggered by CUDA).  It keeps
# every CUDA.jl array, cuBLAS GEMM, attention and DeltaNet path of
# QwenDecisionCoreCUDAExt and replaces only the per-layer row kernels --
# gather, RMSNorm (+ residual), q/k norm + partial RoPE, gated RMSNorm,
# SwiGLU, the attention output gate, the DeltaNet conv + q/k L2 norms and
# its beta / decay gates -- by `ccall`s into libqdc_b200.so
# (include/qdc_b200.h).
#
# Selection.  QwenBackbone(dir; device = :cuda) loads CuArrays exactly as
# before; when the active device is a compute capability 10.0 GPU and the
# library loads, `use_b200()` is true and the hooks below run the sm_100a
# kernels.  The CUDA extension's own kernels are not redefined: its
# `native_*` methods dispatch here through the `B200Kernels` hook table
# that the maintainer adds to ext/cuda_workspace.jl (the call sites are
# listed in the integration notes), so no method is overwritten.
#
# NOTE: Julia is not installed in the environment this library was built
# and tested in; this file is the binding a maintainer adds, exercised there
# only through its Python twin (qdc_b200/_lib.py), which calls the same
# entry points with the same arguments.
module QwenDecisionCoreB200Ext

import QwenDecisionCore
import CUDA

const QDC = QwenDecisionCore
const LIB = get(ENV, "QDC_B200_LIB", joinpath(@__DIR__, "..", "deps", "libqdc_b200.so"))

const QDC_OK = Cint(0)
const QDC_EINVAL = Cint(1)
const QDC_EBOUNDS = Cint(2)
const QDC_F32 = Cint(0)
const QDC_BF16 = Cint(1)

# ---------------------------------------------------------------- context

mutable struct Context
    handle::Ptr{Cvoid}
end

const CONTEXTS = Dict{Int,Context}()
const CONTEXT_LOCK = ReentrantLock()

function check(status::Cint, handle::Ptr{Cvoid} = C_NULL)
    status == QDC_OK && return nothing
    msg = unsafe_string(ccall((:qdc_last_error, LIB), Cstring, (Ptr{Cvoid},), handle))
    isempty(msg) && (msg = unsafe_string(ccall((:qdc_status_string, LIB), Cstring, (Cint,), status)))
    # src/backbone.jl:413-422 raises ArgumentError for bad ids and shapes
    status in (QDC_EINVAL, QDC_EBOUNDS) && throw(ArgumentError(msg))
    error("libqdc_b200: " * msg)
end

function context(dev::CUDA.CuDevice = CUDA.device())
    key = CUDA.deviceid(dev)
    lock(CONTEXT_LOCK) do
        get!(CONTEXTS, key) do
            ref = Ref{Ptr{Cvoid}}(C_NULL)
            check(ccall((:qdc_init, LIB), Cint, (Cint, Ptr{Ptr{Cvoid}}), Cint(key), ref))
            ctx = Context(ref[])
            finalizer(c -> ccall((:qdc_destroy, LIB), Cint, (Ptr{Cvoid},), c.handle), ctx)
            ctx
        end
    end
end

const QDC_B200_ABI_VERSION = Cint(1)

use_b200() = CUDA.functional() && CUDA.capability(CUDA.device()) == v"10.0" && isfile(LIB) &&
             ccall((:qdc_abi_version, LIB), Cint, ()) == QDC_B200_ABI_VERSION

stream_handle() = Base.unsafe_convert(Ptr{Cvoid}, CUDA.stream().handle)
ptr(x::CUDA.CuArray) = Base.unsafe_convert(Ptr{Cvoid}, pointer(x))
ptr(::Nothing) = C_NULL
ld(x::CUDA.CuArray) = Int64(size(x, 1))  # column stride of a dense Julia matrix

# ------------------------------------------------------------- entry points
# Julia (width, tokens) column-major == [tokens][width] row-major: the
# leading dimension of the C ABI is the Julia column stride.

"""residual_rms!(out_r, out_y, x, m, weight, eps; centered=true)

r = x + m (stored in out_r unless it is nothing), y = rms(r) .* (1 .+ w)
(or .* w).  `m === nothing`: plain RMSNorm (src/backbone.jl:200-204)."""
function residual_rms!(out_r, out_y::CUDA.CuArray{Float32}, x::CUDA.CuArray{Float32}, m, weight,
                       eps; centered::Bool = true)
    width = size(x, 1)
    rows = length(x) ÷ width
    ctx = context()
    check(ccall((:qdc_residual_rms, LIB), Cint,
                (Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Cfloat,
                 Cint, Int64, Int64, Int64, Int64, Int64, Int64, Cint, Ptr{Cvoid}),
                ctx.handle, ptr(out_r), ptr(out_y), ptr(x), ptr(m), ptr(weight), Float32(eps),
                Cint(centered), Int64(rows), Int64(width), Int64(width), Int64(width),
                Int64(width), Int64(width), QDC_F32, stream_handle()), ctx.handle)
    return out_y
end

"""gather_rms!(out_x, out_y, embedding, ids, weight, eps)

out_x[:, t] = embedding[:, ids[t]+1]; out_y = rms(out_x) (weight nothing:
gather only).  ids are host integers, validated and staged by the library."""
function gather_rms!(out_x, out_y, embedding::CUDA.CuMatrix{Float32}, ids::Vector{<:Integer},
                     weight, eps)
    hidden, vocab = size(embedding)
    host = Int32.(ids)
    ctx = context()
    check(ccall((:qdc_gather_rms, LIB), Cint,
                (Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Int32}, Ptr{Cvoid}, Ptr{Cvoid},
                 Cfloat, Cint, Int64, Int64, Int64, Cint, Ptr{Cvoid}),
                ctx.handle, ptr(out_x), ptr(out_y), ptr(embedding), host, C_NULL, ptr(weight),
                Float32(eps), Cint(1), Int64(length(host)), Int64(hidden), Int64(vocab), QDC_F32,
                stream_handle()), ctx.handle)
    return out_x, out_y
end

"""qk_norm_rope!(out, projected, weight, eps, rotary, cos, sin; source_width, offset)

Per-head RMSNorm (1+w) and rotate-half RoPE on the first `rotary` dims of
each head of `projected` (head h of token t at rows (h-1)*source_width .+
(1:dim) of column t: source_width = 2dim for the packed [q; gate] query
projection, dim for keys).  `out` is (dim, heads, tokens)."""
function qk_norm_rope!(out::CUDA.CuArray{Float32,3}, projected::CUDA.CuMatrix{Float32}, weight,
                       eps, rotary::Integer, cos::CUDA.CuMatrix{Float32},
                       sin::CUDA.CuMatrix{Float32}; source_width::Integer, offset::Integer = 0)
    dim, heads, tokens = size(out)
    ctx = context()
    check(ccall((:qdc_qk_norm_rope, LIB), Cint,
                (Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Int64, Cint, Cint, Int64, Int64, Ptr{Cvoid},
                 Cfloat, Cint, Ptr{Cvoid}, Ptr{Cvoid}, Int64, Int64, Int64, Ptr{Cvoid}),
                ctx.handle, ptr(out), ptr(projected), Int64(tokens), Cint(heads), Cint(dim),
                Int64(size(projected, 1)), Int64(source_width), ptr(weight), Float32(eps),
                Cint(rotary), ptr(cos), ptr(sin), Int64(size(cos, 2)), Int64(offset), Int64(0),
                stream_handle()), ctx.handle)
    return out
end

"""qk_norm_rope_head_major!(out, projected, weight, eps, rotary, cos, sin;
source_width, row_offset = 0, offset = 0, groups = 1)

qk_norm_rope! writing the head-major (dim, tokens, heads) layout that
prepare_head_kernel! produces and the attention GEMMs read
(ext/cuda_attention.jl:1-45,125-154): out[:, t, h] is head h of token t,
source head h at rows row_offset + (h-1)*source_width .+ (1:dim) of
column t of `projected`.  With groups > 1 the source has heads/groups heads
and each is written to the `groups` query-head slots that read it (query
head h reads kv head cld(h, groups)): one strided launch per slot, as the
reference writes K once per query head.  `offset` is the position of the
first token."""
function qk_norm_rope_head_major!(out::CUDA.CuArray{Float32,3}, projected::CUDA.CuMatrix{Float32}, weight,
                                  eps, rotary::Integer, cos::CUDA.CuMatrix{Float32},
                                  sin::CUDA.CuMatrix{Float32}; source_width::Integer,
                                  row_offset::Integer = 0, offset::Integer = 0, groups::Integer = 1)
    dim, tokens, heads_out = size(out)
    heads = heads_out ÷ groups
    ctx = context()
    for g = 0:groups-1
        check(ccall((:qdc_qk_norm_rope_strided, LIB), Cint,
                    (Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Int64, Cint, Cint, Int64, Int64, Int64, Int64,
                     Ptr{Cvoid}, Cfloat, Cint, Ptr{Cvoid}, Ptr{Cvoid}, Int64, Int64, Int64, Ptr{Cvoid}),
                    ctx.handle, ptr(out) + g * dim * tokens * sizeof(Float32),
                    ptr(projected) + row_offset * sizeof(Float32), Int64(tokens), Cint(heads), Cint(dim),
                    Int64(size(projected, 1)), Int64(source_width), Int64(dim),
                    Int64(groups * dim * tokens), ptr(weight), Float32(eps), Cint(rotary), ptr(cos),
                    ptr(sin), Int64(size(cos, 2)), Int64(offset), Int64(0), stream_handle()), ctx.handle)
    end
    return out
end

const ROPE_DEVICE = Dict{Tuple{Float32,Int,Int},Tuple{CUDA.CuMatrix{Float32},CUDA.CuMatrix{Float32}}}()
const ROPE_LOCK = ReentrantLock()

"""rope_device(theta, rotary, n) -> device (cos, sin) tables of at least n
positions, built once per (theta, rotary, device) and regrown when a longer
sequence arrives."""
function rope_device(theta, rotary::Integer, n::Integer)
    key = (Float32(theta), Int(rotary), CUDA.deviceid(CUDA.device()))
    lock(ROPE_LOCK) do
        hit = get(ROPE_DEVICE, key, nothing)
        if hit === nothing || size(hit[1], 2) < n
            hit = ROPE_DEVICE[key] = rope_tables(Float32(theta), rotary, max(n, 2048))
        end
        hit
    end
end

"""rope_tables(theta, rotary, n) -> (cos, sin) as (rotary/2, n) CuMatrices,
built on the host exactly as src/backbone_cpu.jl:90-105."""
function rope_tables(theta::Float32, rotary::Integer, n::Integer)
    half = rotary ÷ 2
    c = Matrix{Float32}(undef, half, n)
    s = Matrix{Float32}(undef, half, n)
    check(ccall((:qdc_rope_table, LIB), Cint, (Cfloat, Cint, Int64, Ptr{Float32}, Ptr{Float32}),
                theta, Cint(rotary), Int64(n), c, s))
    return CUDA.CuArray(c), CUDA.CuArray(s)
end

"""gated_rms!(out, o, projected, weight, eps; z_offset)

normalized(o) .* w .* silu(z) per (value head, token); z read in place from
rows z_offset .+ (1:heads*dim) of `projected` (ext/cuda_delta.jl:232-241)."""
function gated_rms!(out::CUDA.CuMatrix{Float32}, o::CUDA.CuArray{Float32,3},
                    projected::CUDA.CuMatrix{Float32}, weight, eps; z_offset::Integer)
    dim, heads, tokens = size(o)
    ctx = context()
    check(ccall((:qdc_gated_rms, LIB), Cint,
                (Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Int64, Cint, Cint, Int64, Int64,
                 Int64, Int64, Ptr{Cvoid}, Cfloat, Ptr{Cvoid}),
                ctx.handle, ptr(out), ptr(o), ptr(projected), Int64(tokens), Cint(heads), Cint(dim),
                Int64(dim * heads), Int64(size(projected, 1)), Int64(z_offset), Int64(size(out, 1)),
                ptr(weight), Float32(eps), stream_handle()), ctx.handle)
    return out
end

"""swiglu!(out, packed)  -- out = silu(gate) .* up with gate = packed[1:I, :],
up = packed[I+1:2I, :] (ext/cuda_mlp.jl:63-71)."""
function swiglu!(out::CUDA.CuMatrix{Float32}, packed::CUDA.CuMatrix{Float32})
    width = size(out, 1)
    rows = size(out, 2)
    ctx = context()
    gate = ptr(packed)
    up = gate + width * sizeof(Float32)
    check(ccall((:qdc_swiglu, LIB), Cint,
                (Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Int64, Int64, Int64,
                 Int64, Int64, Ptr{Cvoid}),
                ctx.handle, ptr(out), C_NULL, gate, up, Int64(rows), Int64(width),
                Int64(size(packed, 1)), Int64(size(packed, 1)), Int64(width), stream_handle()),
          ctx.handle)
    return out
end

"""attn_gate!(merged, values, qgate)  -- merged[:, head, token] =
values[:, token, head] .* sigmoid(gate of (head, token)), the gate rows
(head-1)*2dim+dim .+ (1:dim) of the packed [q; gate] projection `qgate`
(merge_gate_kernel!, ext/cuda_attention.jl:92-108).  `values` is the
(dim, tokens, heads) attention output; `merged` is (dim*heads, tokens)."""
function attn_gate!(merged::CUDA.CuMatrix{Float32}, values::CUDA.CuArray{Float32,3},
                    qgate::CUDA.CuMatrix{Float32})
    dim, tokens, heads = size(values)
    ctx = context()
    check(ccall((:qdc_attn_gate, LIB), Cint,
                (Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Int64, Int64, Cint, Cint, Int64,
                 Int64, Int64, Int64, Int64, Int64, Ptr{Cvoid}),
                ctx.handle, ptr(merged), ptr(values), ptr(qgate) + dim * sizeof(Float32),
                Int64(1), Int64(tokens), Cint(heads), Cint(dim), Int64(dim * tokens * heads),
                Int64(dim * tokens), Int64(dim), Int64(size(qgate, 1)), Int64(2 * dim),
                Int64(size(merged, 1)), stream_handle()), ctx.handle)
    return merged
end

"""delta_gates!(beta, decay, projected, a_decay, dt_bias, start)  -- beta =
sigmoid(b), decay = a_decay .* softplus(a .+ dt_bias) for the a rows
start .+ (1:heads) and b rows start+heads .+ (1:heads) of `projected`
(delta_gates_kernel!, ext/cuda_delta.jl:168-181).  beta and decay are
(heads, tokens)."""
function delta_gates!(beta::CUDA.CuMatrix{Float32}, decay::CUDA.CuMatrix{Float32},
                      projected::CUDA.CuMatrix{Float32}, a_decay, dt_bias, start::Integer)
    heads, tokens = size(beta)
    ctx = context()
    check(ccall((:qdc_delta_gates, LIB), Cint,
                (Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Int64, Int64, Ptr{Cvoid}, Ptr{Cvoid},
                 Int64, Cint, Ptr{Cvoid}),
                ctx.handle, ptr(beta), ptr(decay), ptr(projected), Int64(size(projected, 1)),
                Int64(start), ptr(a_decay), ptr(dt_bias), Int64(tokens), Cint(heads),
                stream_handle()), ctx.handle)
    return beta, decay
end

"""delta_conv_norm_mixed!(query, key, mixed, projected, conv, cfg)  --
delta_conv_norm! with v written into rows 2*key_width .+ (1:value_width) of
`mixed` (qkv_width, tokens), where the reference's delta-rule kernels read
it (ext/cuda_delta.jl:199-213); the q and k rows of `mixed` are not
written (the delta rule reads query and key)."""
function delta_conv_norm_mixed!(query::CUDA.CuArray{Float32,3}, key::CUDA.CuArray{Float32,3},
                                mixed::CUDA.CuMatrix{Float32}, projected::CUDA.CuMatrix{Float32},
                                conv::CUDA.CuMatrix{Float32}, cfg)
    tokens = size(projected, 2)
    key_width = cfg.key_dim * cfg.key_heads
    ctx = context()
    check(ccall((:qdc_delta_conv_norm_strided, LIB), Cint,
                (Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Int64, Ptr{Cvoid}, Int64, Ptr{Cvoid},
                 Int64, Int64, Cint, Cint, Cint, Cint, Cfloat, Ptr{Cvoid}),
                ctx.handle, ptr(query), ptr(key), ptr(mixed) + 2 * key_width * sizeof(Float32),
                Int64(size(mixed, 1)), ptr(projected), Int64(size(projected, 1)), ptr(conv),
                Int64(tokens), Int64(0), Cint(cfg.key_heads), Cint(cfg.key_dim), Cint(cfg.value_heads),
                Cint(cfg.value_dim), 1.0f-6, stream_handle()), ctx.handle)
    return query, key, mixed
end

"""delta_conv_norm!(query, key, value, projected, conv, cfg)  -- the causal
4-tap depthwise conv + SiLU of rows 1:qkv_width of `projected`
(causal_depthwise_kernel!, ext/cuda_delta.jl:118-146) followed by the q/k
L2 norms (qk_normalize_kernel!, ext/cuda_delta.jl:8-40) in one pass.
query, key are (key_dim, key_heads, tokens); value is a dense
(value_dim, value_heads, tokens) array, read by the delta rule in place of
rows 2*key_width .+ (1:value_width) of the conv output."""
function delta_conv_norm!(query::CUDA.CuArray{Float32,3}, key::CUDA.CuArray{Float32,3},
                          value::CUDA.CuArray{Float32,3}, projected::CUDA.CuMatrix{Float32},
                          conv::CUDA.CuMatrix{Float32}, cfg)
    tokens = size(projected, 2)
    ctx = context()
    check(ccall((:qdc_delta_conv_norm, LIB), Cint,
                (Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Int64, Ptr{Cvoid}, Int64,
                 Int64, Cint, Cint, Cint, Cint, Cfloat, Ptr{Cvoid}),
                ctx.handle, ptr(query), ptr(key), ptr(value), ptr(projected),
                Int64(size(projected, 1)), ptr(conv), Int64(tokens), Int64(0), Cint(cfg.key_heads),
                Cint(cfg.key_dim), Cint(cfg.value_heads), Cint(cfg.value_dim), 1.0f-6,
                stream_handle()), ctx.handle)
    return query, key, value
end

"""delta_solve!(system, rhs)  -- rhs .= UnitLowerTriangular(system) \\ rhs in place
for one (n, n) system (n <= 64) or a batch (n, n, batch) / (width, n, batch)
-- the delta_solve hook of the chunked gated delta rule (src/backbone.jl:279,
ext/QwenDecisionCoreCUDAExt.jl:22-24) with no solver workspace.  A Julia
column-major (n, n) system is the row-major transpose, so the library sees
rhs' as (n rows x width) and system' as its upper triangle: pass
`transpose`d copies, or use the row-major layout throughout."""
function delta_solve!(system::CUDA.CuArray{Float32}, rhs::CUDA.CuArray{Float32}; n::Integer,
                      width::Integer, batch::Integer = 1)
    ctx = context()
    check(ccall((:qdc_unit_lower_solve, LIB), Cint,
                (Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Int64, Cint, Int64, Int64, Int64, Int64, Int64,
                 Ptr{Cvoid}),
                ctx.handle, ptr(rhs), ptr(system), Int64(batch), Cint(n), Int64(width), Int64(n),
                Int64(n * n), Int64(width), Int64(n * width), stream_handle()), ctx.handle)
    return rhs
end

"""upload_bf16(bits::Array{UInt16}) -> CuArray{Float32}: a checkpoint's raw
BF16 words copied to the device as they are and widened there (bits << 16,
src/safetensors.jl:28-30), half the host -> device bytes of widening on the
host before native_array(::Val{:cuda}, x) (ext/QwenDecisionCoreCUDAExt.jl:7)."""
function upload_bf16(bits::Array{UInt16})
    dev_bits = CUDA.CuArray(bits)
    out = CUDA.CuArray{Float32}(undef, size(bits))
    ctx = context()
    check(ccall((:qdc_bf16_to_f32, LIB), Cint, (Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Int64, Ptr{Cvoid}),
                ctx.handle, ptr(out), ptr(dev_bits), Int64(length(bits)), stream_handle()), ctx.handle)
    return out
end

"""gather!(out, embedding, ids)  -- out[:, t] = embedding[:, ids[t]+1] bit for
bit (native_gather, src/backbone.jl:55-64); host ids validated and staged."""
function gather!(out::CUDA.CuMatrix{Float32}, embedding::CUDA.CuMatrix{Float32}, ids::Vector{<:Integer})
    hidden, vocab = size(embedding)
    host = Int32.(ids)
    ctx = context()
    check(ccall((:qdc_gather, LIB), Cint,
                (Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Int32}, Int64, Int64, Int64, Cint, Ptr{Cvoid}),
                ctx.handle, ptr(out), ptr(embedding), host, Int64(length(host)), Int64(hidden),
                Int64(vocab), QDC_F32, stream_handle()), ctx.handle)
    return out
end

"""gather_rms_device!(out_x, out_y, embedding, ids, weight, eps)  -- gather_rms!
with device ids (a CuVector{Int32}, 0-based), for CUDA-graph capture
(gather_input_kernel!, ext/cuda_io_graph.jl:1-14).  Out-of-range ids poison
their rows and surface as ArgumentError at the next sync!()."""
function gather_rms_device!(out_x, out_y, embedding::CUDA.CuMatrix{Float32}, ids::CUDA.CuVector{Int32},
                            weight, eps)
    hidden, vocab = size(embedding)
    ctx = context()
    check(ccall((:qdc_gather_rms_device_ids, LIB), Cint,
                (Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid},
                 Cfloat, Cint, Int64, Int64, Int64, Cint, Ptr{Cvoid}),
                ctx.handle, ptr(out_x), ptr(out_y), ptr(embedding), ptr(ids), C_NULL, ptr(weight),
                Float32(eps), Cint(1), Int64(length(ids)), Int64(hidden), Int64(vocab), QDC_F32,
                stream_handle()), ctx.handle)
    return out_x, out_y
end

"""gather_rms_noalloc!(out_x, out_y, embedding, ids, weight, eps)  -- gather_rms!
for a host whose memory pool owns every device byte: the library allocates
nothing (no context; ids staged in a fixed 256 KiB array in the library, at
most 65536 per call).  Make the first call on a device at start-up; calls
whose work overlaps on the GPU race on the array, so keep them on one
stream."""
function gather_rms_noalloc!(out_x, out_y, embedding::CUDA.CuMatrix{Float32}, ids::Vector{<:Integer},
                             weight, eps)
    hidden, vocab = size(embedding)
    host = Int32.(ids)
    check(ccall((:qdc_gather_rms_noalloc, LIB), Cint,
                (Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Int32}, Ptr{Cvoid}, Ptr{Cvoid}, Cfloat, Cint,
                 Int64, Int64, Int64, Cint, Ptr{Cvoid}),
                ptr(out_x), ptr(out_y), ptr(embedding), host, C_NULL, ptr(weight), Float32(eps), Cint(1),
                Int64(length(host)), Int64(hidden), Int64(vocab), QDC_F32, stream_handle()))
    return out_x, out_y
end

"""q_k_norm_rope!(q, k, projected, q_norm, k_norm, eps, rotary, cos, sin; q_width, k_offset)

The query heads (first dim of each 2dim-wide [q; gate] head) and the key
heads (rows k_offset .+ (1:dim*kv_heads)) of the packed projection, both
normalised and rotated in one launch (both prepare_head_kernel! launches of
ext/cuda_attention.jl:128,141).  q is (dim, heads, tokens), k is
(dim, kv_heads, tokens)."""
function q_k_norm_rope!(q::CUDA.CuArray{Float32,3}, k::CUDA.CuArray{Float32,3},
                        projected::CUDA.CuMatrix{Float32}, q_norm, k_norm, eps, rotary::Integer,
                        cos::CUDA.CuMatrix{Float32}, sin::CUDA.CuMatrix{Float32}; k_offset::Integer,
                        seq_len::Integer = 0)
    dim, heads, tokens = size(q)
    kv_heads = size(k, 2)
    ld = Int64(size(projected, 1))
    ctx = context()
    check(ccall((:qdc_q_k_norm_rope, LIB), Cint,
                (Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Int64, Cint, Cint, Cint,
                 Int64, Int64, Int64, Int64, Ptr{Cvoid}, Ptr{Cvoid}, Cfloat, Cint, Ptr{Cvoid},
                 Ptr{Cvoid}, Int64, Int64, Int64, Ptr{Cvoid}),
                ctx.handle, ptr(q), ptr(k), ptr(projected), ptr(projected) + k_offset * sizeof(Float32),
                Int64(tokens), Cint(heads), Cint(kv_heads), Cint(dim), ld, Int64(2 * dim), ld,
                Int64(dim), ptr(q_norm), ptr(k_norm), Float32(eps), Cint(rotary), ptr(cos), ptr(sin),
                Int64(size(cos, 2)), Int64(0), Int64(seq_len), stream_handle()), ctx.handle)
    return q, k
end

"""to_bf16!(out::CuArray{UInt16}, x::CuArray{Float32})  -- bf16 storage of x,
round to nearest even by integer add (float32_to_bf16, src/safetensors.jl:38-42)."""
function to_bf16!(out::CUDA.CuArray{UInt16}, x::CUDA.CuArray{Float32})
    length(out) == length(x) || throw(DimensionMismatch("out and x lengths differ"))
    ctx = context()
    check(ccall((:qdc_f32_to_bf16, LIB), Cint, (Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Int64, Ptr{Cvoid}),
                ctx.handle, ptr(out), ptr(x), Int64(length(x)), stream_handle()), ctx.handle)
    return out
end

"""set_pdl!(on::Bool)  -- QDC_OPT_PDL: programmatic dependent launch for this
device's context (on by default)."""
set_pdl!(on::Bool) = check(ccall((:qdc_set_option, LIB), Cint, (Ptr{Cvoid}, Cint, Cint),
                                 context().handle, Cint(1), Cint(on)), context().handle)

# workspace arena (replaces the slot allocator scratch(T, dims),
# ext/cuda_workspace.jl:71-87): reserve once, carve per forward, reset.
ws_reserve!(bytes::Integer) = check(ccall((:qdc_ws_reserve, LIB), Cint, (Ptr{Cvoid}, Csize_t),
                                          context().handle, Csize_t(bytes)), context().handle)
ws_reset!() = check(ccall((:qdc_ws_reset, LIB), Cint, (Ptr{Cvoid},), context().handle), context().handle)

"""ws_mark() / ws_release!(mark) -- the cursor before a layer, and back to it
after: each layer of a kind then carves the same slots in the same order,
as the per-kind slot lists of ext/cuda_workspace.jl:279-300 do."""
function ws_mark()
    ref = Ref{Csize_t}(0)
    check(ccall((:qdc_ws_mark, LIB), Cint, (Ptr{Cvoid}, Ptr{Csize_t}), context().handle, ref),
          context().handle)
    return ref[]
end
ws_release!(mark::Integer) = check(ccall((:qdc_ws_release, LIB), Cint, (Ptr{Cvoid}, Csize_t),
                                         context().handle, Csize_t(mark)), context().handle)

"""ws_stats() -> (used, capacity, high_water) bytes of the arena."""
function ws_stats()
    used, cap, high = Ref{Csize_t}(0), Ref{Csize_t}(0), Ref{Csize_t}(0)
    check(ccall((:qdc_ws_stats, LIB), Cint, (Ptr{Cvoid}, Ptr{Csize_t}, Ptr{Csize_t}, Ptr{Csize_t}),
                context().handle, used, cap, high), context().handle)
    return Int(used[]), Int(cap[]), Int(high[])
end

"""scratch(T, dims...) -> CuArray{T} carved from the context's arena (not owned:
valid until the next ws_reset!())."""
function scratch(::Type{T}, dims::Integer...) where {T}
    ref = Ref{Ptr{Cvoid}}(C_NULL)
    ctx = context()
    check(ccall((:qdc_ws_alloc, LIB), Cint, (Ptr{Cvoid}, Csize_t, Csize_t, Ptr{Ptr{Cvoid}}),
                ctx.handle, Csize_t(prod(dims) * sizeof(T)), Csize_t(256), ref), ctx.handle)
    return unsafe_wrap(CUDA.CuArray, CUDA.CuPtr{T}(UInt(ref[])), dims; own = false)
end

"""sync!() -- the synchronize of native_forward_scope's `finally`
(ext/cuda_workspace.jl:62-66), reporting device-side id errors."""
sync!() = check(ccall((:qdc_sync, LIB), Cint, (Ptr{Cvoid}, Ptr{Cvoid}), context().handle,
                      stream_handle()), context().handle)

# --------------------------------------------------------------- hook table
# ext/cuda_workspace.jl gains `const B200Kernels = Ref{Any}(nothing)` and
# routes its five row-kernel call sites through it when set.
function __init__()
    if use_b200()
        cuda_ext = Base.get_extension(QDC, :QwenDecisionCoreCUDAExt)
        cuda_ext === nothing || (cuda_ext.B200Kernels[] = (; residual_rms!, gather_rms!, gather!,
                                                          gather_rms_device!, gather_rms_noalloc!,
                                                          qk_norm_rope!, qk_norm_rope_head_major!,
                                                          rope_device, delta_conv_norm_mixed!,
                                                          q_k_norm_rope!, rope_tables, gated_rms!,
                                                          swiglu!, attn_gate!, delta_gates!,
                                                          delta_conv_norm!, delta_solve!,
                                                          upload_bf16, to_bf16!,
                                                          set_pdl!, ws_reserve!, ws_reset!,
                                                          ws_mark, ws_release!, ws_stats,
                                                          scratch, sync!))
    end
end

end # module
