"""MetricType with the FAISS integer values.

The reference ships three incompatible enums (python/metalfaiss/metric_type.py:10-21,
python/metalfaiss/types/metric_type.py:8-18); its own test expects the FAISS
integers (python/metalfaiss/unittest/test_metric_type.py:29-40), which is what
this enum uses. Members of the reference's enums (or their names/strings) are
accepted by `MetricType.coerce`, matching by name.
"""
from __future__ import annotations

from enum import IntEnum


class MetricType(IntEnum):
    INNER_PRODUCT = 0
    L2 = 1
    L1 = 2
    LINF = 3
    LP = 4
    CANBERRA = 20
    BRAY_CURTIS = 21
    JENSEN_SHANNON = 22
    JACCARD = 23

    # Aliases used by the reference's string enum (types/metric_type.py).
    Linf = 3
    Canberra = 20
    BrayCurtis = 21
    JensenShannon = 22
    Jaccard = 23

    @classmethod
    def from_string(cls, name: str) -> "MetricType":
        """python/metalfaiss/metric_type.py:22-49, extended with the FAISS spellings."""
        key = name.strip().lower().replace("-", "_").replace(" ", "_")
        table = {
            "inner_product": cls.INNER_PRODUCT, "ip": cls.INNER_PRODUCT,
            "l2": cls.L2, "l1": cls.L1, "linf": cls.LINF, "l_inf": cls.LINF,
            "lp": cls.LP, "canberra": cls.CANBERRA, "bray_curtis": cls.BRAY_CURTIS,
            "braycurtis": cls.BRAY_CURTIS, "jensen_shannon": cls.JENSEN_SHANNON,
            "jensenshannon": cls.JENSEN_SHANNON, "jaccard": cls.JACCARD,
        }
        try:
            return table[key]
        except KeyError:
            raise ValueError(f"Unknown metric type: {name}") from None

    @classmethod
    def coerce(cls, value) -> "MetricType":
        if isinstance(value, MetricType):
            return value
        if isinstance(value, str):
            return cls.from_string(value)
        name = getattr(value, "name", None)
        if isinstance(name, str):  # a member of one of the reference's enums
            return cls.from_string(name)
        return cls(int(value))

    @property
    def is_similarity(self) -> bool:
        return self is MetricType.INNER_PRODUCT

    def __str__(self) -> str:
        return self.name.lower()


SUPPORTED_METRICS = (MetricType.INNER_PRODUCT, MetricType.L2, MetricType.L1, MetricType.LINF)
