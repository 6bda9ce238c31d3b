package com.nablatensor.jax4j.backend.b200;

/** AadEngine "cuda-interp": fixed interpreter kernel over the tape's packed records; engine option "threads". */
public final class B200InterpEngine extends B200AadEngines.Base {
  public B200InterpEngine() {
    super("cuda-interp", 91, B200AadEngines.INTERP, "threads");
  }
}
