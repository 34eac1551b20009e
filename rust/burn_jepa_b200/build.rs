//! Links libbjf.so, the sm_100a library built by burn_jepa_b200/csrc/Makefile.  Set BJF_LIB_DIR to
//! the directory that holds it (the repository's burn_jepa_b200/ after `make`); at run time the
//! loader must find it too (rpath below, or LD_LIBRARY_PATH).
fn main() {
    println!("cargo:rerun-if-env-changed=BJF_LIB_DIR");
    let dir = std::env::var("BJF_LIB_DIR").unwrap_or_else(|_| {
        let here = std::env::var("CARGO_MANIFEST_DIR").expect("cargo sets CARGO_MANIFEST_DIR");
        format!("{here}/../../burn_jepa_b200")
    });
    println!("cargo:rustc-link-search=native={dir}");
    println!("cargo:rustc-link-lib=dylib=bjf");
    println!("cargo:rustc-link-arg=-Wl,-rpath,{dir}");
}
