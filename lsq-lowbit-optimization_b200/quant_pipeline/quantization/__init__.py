from .int4_pack import pack_int4_weights, unpack_int4_weights

__all__ = ["pack_int4_weights", "unpack_int4_weights"]
