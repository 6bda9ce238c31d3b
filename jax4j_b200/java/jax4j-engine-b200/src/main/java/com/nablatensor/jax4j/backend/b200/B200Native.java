package com.nablatensor.jax4j.backend.b200;

import static java.lang.foreign.ValueLayout.ADDRESS;
import static java.lang.foreign.ValueLayout.JAVA_DOUBLE;
import static java.lang.foreign.ValueLayout.JAVA_FLOAT;
import static java.lang.foreign.ValueLayout.JAVA_INT;
import static java.lang.foreign.ValueLayout.JAVA_LONG;

import java.lang.foreign.Arena;
import java.lang.foreign.FunctionDescriptor;
import java.lang.foreign.Linker;
import java.lang.foreign.MemoryLayout;
import java.lang.foreign.MemorySegment;
import java.lang.foreign.SymbolLookup;
import java.lang.invoke.MethodHandle;
import java.nio.file.Path;
import java.util.Map;
import java.util.concurrent.ConcurrentHashMap;

/**
 * Downcalls into libjax4j_b200.so. Every entry point returns an int status (include/jax4j_b200.h):
 * 0 OK, 1 invalid argument, 2 out of memory, 3 CUDA error, 4 unsupported, 5 not initialised,
 * 6 a bounded device wait timed out; {@link #check} maps them to the exceptions the reference's
 * SPI callers expect (IllegalArgumentException, UnsupportedOperationException, ...), with the
 * library's message for the failing call.
 */
public final class B200Native {
  private B200Native() {}

  static final String LIBRARY = System.getProperty("jax4j.b200.lib", "libjax4j_b200.so");
  private static final Linker LINKER = Linker.nativeLinker();
  private static volatile SymbolLookup lookup;
  private static final Map<String, MethodHandle> HANDLES = new ConcurrentHashMap<>();

  /** The library's symbols; loading fails with the loader's message when it is absent. */
  static SymbolLookup lookup() {
    SymbolLookup l = lookup;
    if (l == null) {
      synchronized (B200Native.class) {
        if (lookup == null) {
          lookup = LIBRARY.contains("/")
              ? SymbolLookup.libraryLookup(Path.of(LIBRARY), Arena.global())
              : SymbolLookup.libraryLookup(LIBRARY, Arena.global());
        }
        l = lookup;
      }
    }
    return l;
  }

  /** Downcall handle of an int-returning entry point with the given argument layouts. */
  static MethodHandle fn(String name, MemoryLayout... args) {
    return HANDLES.computeIfAbsent(name, n -> LINKER.downcallHandle(
        lookup().find(n).orElseThrow(() -> new UnsatisfiedLinkError(n + " not found in " + LIBRARY)),
        FunctionDescriptor.of(JAVA_INT, args)));
  }

  /** Calls an entry point and checks its status. */
  static void call(String name, MemoryLayout[] layouts, Object... args) {
    int status;
    try {
      status = (int) fn(name, layouts).invokeWithArguments(args);
    } catch (RuntimeException | Error e) {
      throw e;
    } catch (Throwable t) {
      throw new IllegalStateException(name + " failed", t);
    }
    check(status, name);
  }

  static MemoryLayout[] sig(MemoryLayout... layouts) {
    return layouts;
  }

  static final MemoryLayout P = ADDRESS, L = JAVA_LONG, I = JAVA_INT, F = JAVA_FLOAT, D = JAVA_DOUBLE;

  static void check(int status, String what) {
    if (status == 0) return;
    String msg = lastError(what);
    switch (status) {
      case 1 -> throw new IllegalArgumentException(msg);
      case 2 -> throw new OutOfMemoryError(msg);
      case 4 -> throw new UnsupportedOperationException(msg);
      default -> throw new IllegalStateException(what + " failed: " + msg);
    }
  }

  static String lastError(String fallback) {
    try (Arena a = Arena.ofConfined()) {
      MemorySegment buf = a.allocate(1024);
      int st = (int) fn("j4b_last_error", ADDRESS, JAVA_LONG).invokeExact(buf, 1024L);
      String s = buf.getString(0);
      return st == 0 && !s.isEmpty() ? s : fallback;
    } catch (Throwable t) {
      return fallback;
    }
  }

  /** j4b_free from a cleaner or release: stream-ordered, best effort, never throws. */
  static void free(long address) {
    try {
      int st = (int) fn("j4b_free", JAVA_LONG).invokeExact(address);
    } catch (Throwable ignored) {
      // the process is shutting down or the library is gone; nothing left to free
    }
  }

  static void quantFree(MemorySegment handle) {
    try {
      int st = (int) fn("j4b_quant_free", ADDRESS).invokeExact(handle);
    } catch (Throwable ignored) {
      // as free()
    }
  }

  /** Number of usable GPUs; 0 when the library or a GPU is missing. Never throws. */
  static int deviceCount() {
    try (Arena a = Arena.ofConfined()) {
      MemorySegment n = a.allocate(JAVA_INT);
      int st = (int) fn("j4b_device_count", ADDRESS).invokeExact(n);
      return st == 0 ? n.get(JAVA_INT, 0) : 0;
    } catch (Throwable t) {
      return 0;
    }
  }
}
