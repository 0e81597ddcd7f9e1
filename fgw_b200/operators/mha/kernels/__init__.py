"""Launch layers over libfgw_mha.so."""
