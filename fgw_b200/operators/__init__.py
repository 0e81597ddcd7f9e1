"""Drop-in counterpart of FGW's ``operators`` package for B200."""
