package com.nablatensor.jax4j.backend.b200;

/** AadEngine "cuda": per-tape generated kernel (NVRTC), forward and reverse sweeps fully unrolled. */
public final class B200AadEngine extends B200AadEngines.Base {
  public B200AadEngine() {
    super("cuda", 101, B200AadEngines.GENERATED, null);
  }
}
