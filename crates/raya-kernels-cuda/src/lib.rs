//! raya's `AttentionKernel` on NVIDIA B200 (sm_100a): a thin binding of the
//! C ABI of libraya_attn (`include/raya_attn.h` of the raya_b200 repository).
//!
//! * [`Cuda`] is the drop-in kernel for the trait of
//!   `crates/raya-kernels/src/attention.rs:113-125`: host slices in, the host
//!   slice `out` filled, synchronous, the reference's three error kinds
//!   (`raya_attn_forward_host`).  It runs every mask the encoder asks for:
//!   `Block3`, `Window64`, `Sliding(w)` and `Full`.
//! * [`MultiCuda`] runs one call over several GPUs of this process: the
//!   heads are cut into contiguous ranges balanced by allowed query/key
//!   pairs, one per device, all at once (`raya_attn_forward_multi_gpu`).
//!
//! Errors come back as data (`raya_attn_last_error_info`), so
//! `KernelError::Length { name, got, expected }` is rebuilt without reading
//! the message.  Failures with no reference counterpart (a CUDA call that
//! failed, a device-side wait that gave up) are reported as
//! `KernelError::Unsupported` with the library's message, which starts with
//! `cuda:` or `timeout:`.

use std::ffi::CStr;
use std::os::raw::{c_char, c_int};
use std::ptr;

use raya_kernels::{AttentionKernel, AttnParams, AttnShape, KernelError, Mask};

/// `raya_attn_desc`: the shape and parameters of one call.
#[repr(C)]
#[derive(Debug, Clone, Copy)]
struct RayaAttnDesc {
    batch: i64,
    heads: i64,
    seq: i64,
    head_dim: i64,
    block: i64,
    mask: i32,
    halo: i32,
    window: i64,
    scale: f32,
}

// raya_attn_status and raya_mask_kind values.
const STATUS_OK: c_int = 0;
const STATUS_SHAPE: c_int = 1;
const STATUS_LENGTH: c_int = 2;
const STATUS_UNSUPPORTED: c_int = 3;
const MASK_BLOCK: i32 = 0;
const MASK_WINDOW: i32 = 1;
const MASK_FULL: i32 = 2;

extern "C" {
    fn raya_attn_forward_host(
        desc: *const RayaAttnDesc,
        q: *const f32,
        q_len: usize,
        k: *const f32,
        k_len: usize,
        v: *const f32,
        v_len: usize,
        out: *mut f32,
        out_len: usize,
        valid_len: *const i32,
        device: c_int,
    ) -> c_int;
    fn raya_attn_forward_multi_gpu(
        desc: *const RayaAttnDesc,
        q: *const f32,
        q_len: usize,
        k: *const f32,
        k_len: usize,
        v: *const f32,
        v_len: usize,
        out: *mut f32,
        out_len: usize,
        valid_len: *const i32,
        devices: *const c_int,
        ndevices: c_int,
        out_device0: *mut f32,
    ) -> c_int;
    fn raya_attn_last_error() -> *const c_char;
    fn raya_attn_last_error_info(
        kind: *mut c_int,
        name: *mut *const c_char,
        got: *mut usize,
        expected: *mut usize,
    ) -> c_int;
}

fn to_i64(x: usize, what: &str) -> Result<i64, KernelError> {
    i64::try_from(x).map_err(|_| KernelError::Shape(format!("{what} {x} is out of range")))
}

/// The reference's one-sequence call as the library's descriptor (batch 1):
/// Block3 is the BLOCK mask with one block of halo, Window64 and Sliding(w)
/// the WINDOW mask of half width 64 or w, Full the FULL mask.
fn descriptor(shape: AttnShape, params: &AttnParams) -> Result<RayaAttnDesc, KernelError> {
    let (mask, halo, window) = match params.mask {
        Mask::Block3 => (MASK_BLOCK, 1, 0),
        Mask::Window64 => (MASK_WINDOW, 0, to_i64(raya_kernels::WINDOW, "window")?),
        Mask::Sliding(w) => (MASK_WINDOW, 0, to_i64(w, "window")?),
        Mask::Full => (MASK_FULL, 0, 0),
    };
    Ok(RayaAttnDesc {
        batch: 1,
        heads: to_i64(shape.heads, "heads")?,
        seq: to_i64(shape.seq, "seq")?,
        head_dim: to_i64(shape.head_dim, "head_dim")?,
        block: to_i64(params.block, "block")?,
        mask,
        halo,
        window,
        scale: params.scale,
    })
}

/// The one valid length of the call; one past i32 exceeds every supported seq.
fn valid_len(shape: AttnShape, params: &AttnParams) -> Result<i32, KernelError> {
    i32::try_from(params.valid_len).map_err(|_| {
        KernelError::Shape(format!("valid_len {} exceeds seq {}", params.valid_len, shape.seq))
    })
}

/// The buffer names the library reports, as the `&'static str` the
/// reference's `KernelError::Length` holds.
fn static_name(name: &str) -> &'static str {
    match name {
        "q" => "q",
        "k" => "k",
        "v" => "v",
        "out" => "out",
        "workspace" => "workspace",
        _ => "buffer",
    }
}

/// The error the library raised on this thread, as the reference's type.
fn last_error(status: c_int) -> KernelError {
    // SAFETY: the library returns a NUL-terminated, thread-local string that
    // stays valid until this thread's next failing call.
    let msg = unsafe { CStr::from_ptr(raya_attn_last_error()) }.to_string_lossy().into_owned();
    let strip = |prefix: &str| msg.strip_prefix(prefix).unwrap_or(&msg).to_string();
    match status {
        STATUS_SHAPE => KernelError::Shape(strip("invalid shape: ")),
        STATUS_LENGTH => {
            let mut kind: c_int = 0;
            let mut name: *const c_char = ptr::null();
            let mut got: usize = 0;
            let mut expected: usize = 0;
            // SAFETY: every pointer is a valid local; the call only writes them.
            unsafe { raya_attn_last_error_info(&mut kind, &mut name, &mut got, &mut expected) };
            let name = if name.is_null() {
                ""
            } else {
                // SAFETY: a NUL-terminated thread-local string, as above.
                unsafe { CStr::from_ptr(name) }.to_str().unwrap_or("")
            };
            KernelError::Length { name: static_name(name), got, expected }
        }
        STATUS_UNSUPPORTED => KernelError::Unsupported(strip("unsupported: ")),
        _ => KernelError::Unsupported(msg),
    }
}

fn check(status: c_int) -> Result<(), KernelError> {
    if status == STATUS_OK {
        Ok(())
    } else {
        Err(last_error(status))
    }
}

/// The B200 kernel behind raya's trait, on GPU `device`: the same contract
/// as `Naive` and `Tiled` (host slices, synchronous).  Thread-safe: calls on
/// one device serialise on its staging buffers.
#[derive(Debug, Clone, Copy, Default, PartialEq, Eq)]
pub struct Cuda {
    pub device: i32,
}

impl AttentionKernel for Cuda {
    fn name(&self) -> &'static str {
        "cuda-b200"
    }

    fn attend(
        &self,
        shape: AttnShape,
        params: AttnParams,
        q: &[f32],
        k: &[f32],
        v: &[f32],
        out: &mut [f32],
    ) -> Result<(), KernelError> {
        let d = descriptor(shape, &params)?;
        let valid = valid_len(shape, &params)?;
        // SAFETY: the slices are valid for their lengths, which the library
        // checks against the shape before reading or writing; `out` is
        // borrowed mutably for the duration of the synchronous call.
        check(unsafe {
            raya_attn_forward_host(
                &d,
                q.as_ptr(),
                q.len(),
                k.as_ptr(),
                k.len(),
                v.as_ptr(),
                v.len(),
                out.as_mut_ptr(),
                out.len(),
                &valid,
                self.device,
            )
        })
    }
}

/// One call over several GPUs of this process (distinct device ids): the
/// heads are split into contiguous ranges balanced by allowed pairs, each
/// device runs its range, and every device's part lands in `out`.  The
/// result is bit-identical to [`Cuda`] on one device.
#[derive(Debug, Clone, PartialEq, Eq)]
pub struct MultiCuda {
    pub devices: Vec<i32>,
}

impl AttentionKernel for MultiCuda {
    fn name(&self) -> &'static str {
        "cuda-b200-multi"
    }

    fn attend(
        &self,
        shape: AttnShape,
        params: AttnParams,
        q: &[f32],
        k: &[f32],
        v: &[f32],
        out: &mut [f32],
    ) -> Result<(), KernelError> {
        let d = descriptor(shape, &params)?;
        let valid = valid_len(shape, &params)?;
        let n = c_int::try_from(self.devices.len())
            .map_err(|_| KernelError::Shape(format!("{} devices", self.devices.len())))?;
        // SAFETY: as for `Cuda::attend`; `devices` is valid for `n` ids.
        check(unsafe {
            raya_attn_forward_multi_gpu(
                &d,
                q.as_ptr(),
                q.len(),
                k.as_ptr(),
                k.len(),
                v.as_ptr(),
                v.len(),
                out.as_mut_ptr(),
                out.len(),
                &valid,
                self.devices.as_ptr(),
                n,
                ptr::null_mut(),
            )
        })
    }
}

#[cfg(test)]
mod tests {
    //! Argument checks run before any device work, so these need the library
    //! but not a GPU (tests/oracle.rs:35-78 of raya-kernels, through the FFI).
    use super::*;

    fn shape() -> AttnShape {
        AttnShape { heads: 1, seq: 4, head_dim: 8 }
    }

    #[test]
    fn length_errors_carry_their_fields() {
        let p = AttnParams::new(Mask::Block3, 4, 8);
        let ok = vec![0.0f32; 32];
        let mut out = vec![0.0f32; 32];
        let err = Cuda::default().attend(shape(), p, &ok[..3], &ok, &ok, &mut out).unwrap_err();
        assert_eq!(err, KernelError::Length { name: "q", got: 3, expected: 32 });
        assert_eq!(err.to_string(), "buffer `q` has length 3, expected 32");
        let mut short = vec![0.0f32; 5];
        let err = Cuda::default().attend(shape(), p, &ok, &ok, &ok, &mut short).unwrap_err();
        assert_eq!(err, KernelError::Length { name: "out", got: 5, expected: 32 });
    }

    #[test]
    fn shape_errors_keep_the_reference_text() {
        let ok = vec![0.0f32; 32];
        let mut out = vec![0.0f32; 32];
        let bad = AttnShape { heads: 1, seq: 4, head_dim: 12 };
        let buf = vec![0.0f32; 48];
        let mut out12 = vec![0.0f32; 48];
        let err = Cuda::default()
            .attend(bad, AttnParams::new(Mask::Block3, 4, 12), &buf, &buf, &buf, &mut out12)
            .unwrap_err();
        assert_eq!(err.to_string(), "invalid shape: head_dim 12 is not a multiple of 8");
        let err = Cuda::default()
            .attend(shape(), AttnParams::new(Mask::Block3, 5, 8), &ok, &ok, &ok, &mut out)
            .unwrap_err();
        assert_eq!(err.to_string(), "invalid shape: valid_len 5 exceeds seq 4");
    }

    #[test]
    fn multi_gpu_rejects_repeated_devices() {
        let ok = vec![0.0f32; 32];
        let mut out = vec![0.0f32; 32];
        let err = MultiCuda { devices: vec![0, 0] }
            .attend(shape(), AttnParams::new(Mask::Block3, 4, 8), &ok, &ok, &ok, &mut out)
            .unwrap_err();
        assert!(matches!(err, KernelError::Shape(ref m) if m.contains("listed twice")), "{err}");
    }
}
