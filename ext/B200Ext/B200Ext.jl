# B200Ext -- the JLUST package extension that runs JLUST's sparse hot path on
# libjlust_b200.so (hand-written sm_100a CUDA behind a C ABI).
#
# Drop this directory into JLUST's ext/ and register it in Project.toml's
# [extensions] as `B200Ext = "CUDA"`; set ENV["JLUST_B200_LIB"] (or place the
# library under deps/) to the built libjlust_b200.so.  JLUST itself is not
# modified: the extension adds a third backend next to EmitterBackend and
# CUSPARSEBackend (src/backends.jl:171-181) and a default_backend policy for
# CuArray-backed tensors (as ext/CUDAExt/CUDAExt.jl:232-241 does).
#
# Every ccall below passes exactly the argument list declared for the entry
# point in include/jlust_b200.h (the Python mirror in jlust_b200/_lib.py
# declares the same lists; tests/test_julia_binding.py checks this file's
# ccall signatures against the header).
module B200Ext

using JLUST, CUDA
import JLUST: USTensor, Op, execute, prepare, update_values!, supports_backend,
              positions, coordinates, nonzeros, extents, index_origin, OneBased,
              format_family, AbstractKernelHandle

const lib = get(ENV, "JLUST_B200_LIB",
                joinpath(@__DIR__, "..", "..", "deps", "libjlust_b200.so"))

struct B200Backend <: JLUST.AbstractUSTBackend end

"""A bounded device-side wait gave up (status 10, JLB_ERR_DEVICE_TIMEOUT): the
multi-GPU halo iteration waited for a neighbour that did not publish.  JLUST
has no exception for it."""
struct B200DeviceTimeout <: Exception
    msg::String
end
Base.showerror(io::IO, e::B200DeviceTimeout) = print(io, "B200DeviceTimeout: ", e.msg)

# value / order / mode enums (include/jlust_b200.h)
_dt(::Type{Float32}) = Cint(0)
_dt(::Type{Float64}) = Cint(1)
_dt(::Type{T}) where {T} = throw(JLUST.UnsupportedValueType(T, B200Backend()))
_base(u) = index_origin(u) isa OneBased ? Cint(1) : Cint(0)
_stream() = CUDA.stream().handle
_order(A::CuMatrix) = (Cint(1), Int64(max(stride(A, 2), 1)))          # column-major
_order(A::Transpose{<:Any,<:CuMatrix}) = (Cint(0), Int64(max(stride(parent(A), 2), 1)))

# status codes -> src/errors.jl exceptions (1-7), the others as errors
function _check(st::Cint, be=B200Backend())
    st == 0 && return nothing
    buf = Vector{UInt8}(undef, 512)
    ccall((:jlb_last_error, lib), Cint, (Ptr{UInt8}, Csize_t), buf, length(buf))
    msg = unsafe_string(pointer(buf))
    st == 1 && throw(JLUST.UnsupportedFormat(msg, be))
    st == 2 && throw(JLUST.UnsupportedIndexType(Int32, be))
    st == 3 && throw(JLUST.UnsupportedValueType(Any, be))
    st == 4 && throw(JLUST.IndexOriginMismatch(msg, "idx_base 0 or 1 on every buffer"))
    st == 5 && throw(JLUST.DeviceMismatch(msg))
    st == 6 && throw(JLUST.IncompatibleExtents(msg))
    st == 7 && throw(JLUST.NonCanonicalStorage(msg))
    st == 10 && throw(B200DeviceTimeout(msg))
    error("libjlust_b200 (status $st): " * msg)   # 8 invalid argument, 9 CUDA, 11 workspace
end

supports_backend(::B200Backend, ::Op{:SpMV, Tuple{A,X,Y}}) where {A,X,Y} =
    format_family(A) in (:CSR, :DCSR, :COO, :CSC) &&
    format_family(X) === :Dense && format_family(Y) === :Dense
supports_backend(::B200Backend, ::Op{:SpMM, Tuple{A,B,C}}) where {A,B,C} =
    format_family(A) in (:CSR, :BSR) && format_family(B) === :Dense && format_family(C) === :Dense
supports_backend(::B200Backend, ::Op{:SDDMM, Tuple{A,B,C}}) where {A,B,C} =
    format_family(A) === :Dense && format_family(B) === :Dense && format_family(C) === :CSR

# ----------------------------------------------------------------- SpMV
# replaces execute(::EmitterBackend, ::Op{:SpMV}) (KA spmv.jl:371-504)
function execute(::B200Backend, ::Op{:SpMV,F}, A::USTensor, x::USTensor, y::USTensor;
                 alpha=one(eltype(A)), beta=zero(eltype(A)),
                 input_fn=identity, output_fn=identity) where {F}
    (input_fn === identity && output_fn === identity) ||
        throw(JLUST.UnsupportedFormat(JLUST.format(A), B200Backend()))  # closures cannot cross the ABI
    m, n = extents(A)
    fam = format_family(A)
    if fam === :CSR
        st = ccall((:jlb_csr_spmv, lib), Cint,
                   (Ptr{Cvoid}, Cint, Cint, Int64, Int64, Int64, CuPtr{Int32}, CuPtr{Int32},
                    CuPtr{Cvoid}, CuPtr{Cvoid}, CuPtr{Cvoid}, Cdouble, Cdouble),
                   _stream(), _dt(eltype(A)), _base(A), m, n, length(nonzeros(A)),
                   positions(A, 2), coordinates(A, 2), nonzeros(A), nonzeros(x), nonzeros(y),
                   alpha, beta)
    elseif fam === :DCSR
        st = ccall((:jlb_dcsr_spmv, lib), Cint,
                   (Ptr{Cvoid}, Cint, Cint, Int64, Int64, Int64, Int64, CuPtr{Int32},
                    CuPtr{Int32}, CuPtr{Int32}, CuPtr{Cvoid}, CuPtr{Cvoid}, CuPtr{Cvoid},
                    Cdouble, Cdouble),
                   _stream(), _dt(eltype(A)), _base(A), m, n, length(coordinates(A, 1)),
                   length(nonzeros(A)), positions(A, 2), coordinates(A, 1), coordinates(A, 2),
                   nonzeros(A), nonzeros(x), nonzeros(y), alpha, beta)
    elseif fam === :COO
        st = ccall((:jlb_coo_spmv, lib), Cint,
                   (Ptr{Cvoid}, Cint, Cint, Int64, Int64, Int64, CuPtr{Int32}, CuPtr{Int32},
                    CuPtr{Cvoid}, CuPtr{Cvoid}, CuPtr{Cvoid}, Cdouble, Cdouble),
                   _stream(), _dt(eltype(A)), _base(A), m, n, length(nonzeros(A)),
                   coordinates(A, 1), coordinates(A, 2), nonzeros(A), nonzeros(x), nonzeros(y),
                   alpha, beta)
    elseif fam === :CSC
        st = ccall((:jlb_csc_spmv, lib), Cint,
                   (Ptr{Cvoid}, Cint, Cint, Int64, Int64, Int64, CuPtr{Int32}, CuPtr{Int32},
                    CuPtr{Cvoid}, CuPtr{Cvoid}, CuPtr{Cvoid}, Cdouble, Cdouble),
                   _stream(), _dt(eltype(A)), _base(A), m, n, length(nonzeros(A)),
                   positions(A, 2), coordinates(A, 2), nonzeros(A), nonzeros(x), nonzeros(y),
                   alpha, beta)
    else
        throw(JLUST.UnsupportedFormat(JLUST.format(A), B200Backend()))
    end
    _check(st); y
end

# ----------------------------------------------------------------- SpMM
# replaces the CUSPARSEBackend SpMM default (CUDAExt/ops/spmm.jl:50-58).
# Column-major B and C (JLUST's native layout) go through row-major copies in
# a workspace the library transposes on the stream.
function execute(::B200Backend, ::Op{:SpMM,F}, A::USTensor, B::USTensor, C::USTensor;
                 alpha=one(eltype(A)), beta=zero(eltype(A))) where {F}
    format_family(A) === :BSR && return _bsr_spmm(A, B, C, alpha, beta)
    m, n = extents(A); k = size(nonzeros(B), 2)
    bo, ldb = _order(nonzeros(B)); co, ldc = _order(nonzeros(C))
    wsb = ccall((:jlb_csr_spmm_workspace_size, lib), Csize_t,
                (Cint, Int64, Int64, Int64, Cint, Cint), _dt(eltype(A)), m, n, k, bo, co)
    ws = CuArray{UInt8}(undef, Int(wsb))
    st = ccall((:jlb_csr_spmm_ws, lib), Cint,
               (Ptr{Cvoid}, Cint, Cint, Int64, Int64, Int64, CuPtr{Int32}, CuPtr{Int32},
                CuPtr{Cvoid}, Int64, CuPtr{Cvoid}, Int64, Cint, CuPtr{Cvoid}, Int64, Cint,
                Cdouble, Cdouble, CuPtr{Cvoid}, Csize_t),
               _stream(), _dt(eltype(A)), _base(A), m, n, length(nonzeros(A)),
               positions(A, 2), coordinates(A, 2), nonzeros(A), k, nonzeros(B), ldb, bo,
               nonzeros(C), ldc, co, alpha, beta, ws, wsb)
    _check(st); C
end

# BSR SpMM on tcgen05 tensor cores: BSRRight((64, 64)) BFloat16 values, B
# BFloat16 row-major, C Float32 row-major (src/block_sparse.jl:284-302)
function _bsr_spmm(A::USTensor, B::USTensor, C::USTensor, alpha, beta)
    b1, b2 = JLUST.block_size(JLUST.format(A))
    b1 == b2 || throw(JLUST.UnsupportedFormat(JLUST.format(A), B200Backend()))
    m, n = extents(A); N = size(nonzeros(C), 2)
    _, ldb = _order(nonzeros(B)); _, ldc = _order(nonzeros(C))
    st = ccall((:jlb_bsr_spmm, lib), Cint,
               (Ptr{Cvoid}, Cint, Int64, Int64, Int64, Cint, CuPtr{Int32}, CuPtr{Int32},
                CuPtr{Cvoid}, Int64, CuPtr{Cvoid}, Int64, CuPtr{Float32}, Int64, Cdouble, Cdouble),
               _stream(), _base(A), cld(m, b1), cld(n, b1), length(coordinates(A, 2)), b1,
               positions(A, 2), coordinates(A, 2), nonzeros(A), N, nonzeros(B), ldb,
               nonzeros(C), ldc, alpha, beta)
    _check(st); C
end

# ---------------------------------------------------------------- SDDMM
# mode 0 = the reference's additive form (KA sddmm.jl:23-36): column-major A
# and the column-major K x n B are the fast layouts
function execute(::B200Backend, ::Op{:SDDMM,F}, A::USTensor, B::USTensor, C::USTensor;
                 alpha=one(eltype(C)), beta=zero(eltype(C))) where {F}
    m, n = extents(C); K = size(nonzeros(A), 2)
    ao, lda = _order(nonzeros(A)); bo, ldb = _order(nonzeros(B))
    st = ccall((:jlb_sddmm, lib), Cint,
               (Ptr{Cvoid}, Cint, Cint, Int64, Int64, Int64, CuPtr{Int32}, CuPtr{Int32},
                Int64, CuPtr{Cvoid}, Int64, Cint, CuPtr{Cvoid}, Int64, Cint, CuPtr{Cvoid},
                CuPtr{Cvoid}, Cint, Cdouble, Cdouble),
               _stream(), _dt(eltype(C)), _base(C), m, n, length(nonzeros(C)),
               positions(C, 2), coordinates(C, 2), K, nonzeros(A), lda, ao, nonzeros(B), ldb, bo,
               CU_NULL, nonzeros(C), Cint(0), alpha, beta)
    _check(st); C
end

# ------------------------------------------------- prepare / update_values!
# src/ops.jl:164-188; EmitterSpMVHandle (KA spmv.jl:518-544)
mutable struct B200SpMVHandle{T} <: AbstractKernelHandle
    plan::Ptr{Cvoid}
    A::USTensor
end
function prepare(::B200Backend, ::Type{<:Op{:SpMV}}, A::USTensor{T}) where {T}
    p = Ref{Ptr{Cvoid}}(C_NULL); m, n = extents(A)
    _check(ccall((:jlb_spmv_plan_create, lib), Cint,
                 (Ref{Ptr{Cvoid}}, Ptr{Cvoid}, Cint, Cint, Int64, Int64, Int64,
                  CuPtr{Int32}, CuPtr{Int32}),
                 p, _stream(), _dt(T), _base(A), m, n, length(nonzeros(A)),
                 positions(A, 2), coordinates(A, 2)))
    h = B200SpMVHandle{T}(p[], A)
    finalizer(h -> ccall((:jlb_spmv_plan_destroy, lib), Cint, (Ptr{Cvoid},), h.plan), h)
end
function execute(h::B200SpMVHandle, x::USTensor, y::USTensor; alpha=1.0, beta=0.0)
    _check(ccall((:jlb_spmv_plan_execute, lib), Cint,
                 (Ptr{Cvoid}, Ptr{Cvoid}, CuPtr{Cvoid}, CuPtr{Cvoid}, CuPtr{Cvoid}, Cdouble,
                  Cdouble),
                 h.plan, _stream(), nonzeros(h.A), nonzeros(x), nonzeros(y), alpha, beta))
    y
end
update_values!(h::B200SpMVHandle, A::USTensor) = (h.A = A; h)

# ------------------------------------------------------------ conversions
# convert_format(u, BSRRight((b, b))) for CuArray-backed CSR
# (src/convert.jl:302-388): count phase (block row pointer, nnzb), then fill
function csr_to_bsr(A::USTensor{T}, b::Int) where {T}
    m, n = extents(A); nnz = length(nonzeros(A))
    dt = T === Float32 ? Cint(0) : T === Float64 ? Cint(1) : Cint(2)
    wsb = ccall((:jlb_csr_to_bsr_workspace_size, lib), Csize_t,
                (Int64, Int64, Int64, Cint, Cint), m, n, nnz, b, b)
    ws = CuArray{UInt8}(undef, Int(wsb))
    browptr = CuArray{Int32}(undef, cld(m, b) + 1)
    nnzb = Ref{Int64}(0)
    _check(ccall((:jlb_csr_to_bsr_count, lib), Cint,
                 (Ptr{Cvoid}, Cint, Cint, Int64, Int64, Int64, CuPtr{Int32}, CuPtr{Int32},
                  CuPtr{Cvoid}, Cint, Cint, CuPtr{Int32}, Ref{Int64}, CuPtr{Cvoid}, Csize_t),
                 _stream(), dt, _base(A), m, n, nnz, positions(A, 2), coordinates(A, 2),
                 nonzeros(A), b, b, browptr, nnzb, ws, wsb))
    bcolind = CuArray{Int32}(undef, nnzb[])
    bval = CuArray{T}(undef, nnzb[] * b * b)
    _check(ccall((:jlb_csr_to_bsr_fill, lib), Cint,
                 (Ptr{Cvoid}, Cint, Cint, Int64, Int64, Int64, CuPtr{Int32}, CuPtr{Int32},
                  CuPtr{Cvoid}, Cint, Cint, CuPtr{Int32}, Int64, CuPtr{Int32}, CuPtr{Cvoid},
                  CuPtr{Cvoid}, Csize_t),
                 _stream(), dt, _base(A), m, n, nnz, positions(A, 2), coordinates(A, 2),
                 nonzeros(A), b, b, browptr, nnzb[], bcolind, bval, ws, wsb))
    browptr, bcolind, bval
end

# exclusive scan of Int32 counts into a position buffer (src/convert.jl:154-168)
function exclusive_scan!(out::CuVector{Int32}, counts::CuVector{Int32}, base::Integer)
    n = length(counts)
    wsb = ccall((:jlb_scan_workspace_size, lib), Csize_t, (Int64,), n)
    ws = CuArray{UInt8}(undef, Int(wsb))
    _check(ccall((:jlb_exclusive_scan_i32, lib), Cint,
                 (Ptr{Cvoid}, Int64, CuPtr{Int32}, CuPtr{Int32}, Cint, CuPtr{Cvoid}, Csize_t),
                 _stream(), n, counts, out, Cint(base), ws, wsb))
    out
end

# the same without any allocation, for finalizers and allocator callbacks
# (at most JLB_SCAN_NOALLOC_MAX_N counts; calls on one GPU must not overlap)
exclusive_scan_noalloc!(out::CuVector{Int32}, counts::CuVector{Int32}, base::Integer) =
    (_check(ccall((:jlb_exclusive_scan_i32_noalloc, lib), Cint,
                  (Ptr{Cvoid}, Int64, CuPtr{Int32}, CuPtr{Int32}, Cint),
                  _stream(), length(counts), counts, out, Cint(base))); out)

# --------------------------------------------------------- the drop-in policy
const _CuUST = USTensor{T,I,N,VA} where {T,I,N,VA<:CuArray}
JLUST.default_backend(::_CuUST, ::Type{<:Op{:SpMV}})  = B200Backend()
JLUST.default_backend(::_CuUST, ::Type{<:Op{:SpMM}})  = B200Backend()
JLUST.default_backend(::_CuUST, ::Type{<:Op{:SDDMM}}) = B200Backend()

end # module
